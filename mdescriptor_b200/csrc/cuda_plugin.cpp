// `mdescriptor._cuda` drop-in plugin: the Python-visible ABI that MDescriptor's
// lazy CUDA seam loads (src/mdescriptor/_runtime.py:78-125 via
// MDESCRIPTOR_CUDA_PLUGIN_DIR, src/mdescriptor/_cuda_loader.py), implemented as
// a thin pybind11 layer over the C ABI of libmdsoap (include/mdsoap.h).
//
// Mirrors cpp/cuda/src/bindings.cu:15-57 (module attributes, exception
// registration, create_backend) and the SOAP parts of Backend
// (cpp/cuda/src/backend.cu:296-356, 570-588, 720-744) and
// compute_soap_descriptor's option parsing and result dictionary
// (cpp/cuda/src/extended_descriptors_soap.cuh:806-906, 1115-1124).
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdlib>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/mdsoap.h"

namespace py = pybind11;

namespace {

// Element symbols by atomic number (1..118), for species-keyed option maps.
constexpr const char* kElementSymbols[118] = {
    "H",  "He", "Li", "Be", "B",  "C",  "N",  "O",  "F",  "Ne", "Na", "Mg", "Al", "Si", "P",  "S",  "Cl", "Ar",
    "K",  "Ca", "Sc", "Ti", "V",  "Cr", "Mn", "Fe", "Co", "Ni", "Cu", "Zn", "Ga", "Ge", "As", "Se", "Br", "Kr",
    "Rb", "Sr", "Y",  "Zr", "Nb", "Mo", "Tc", "Ru", "Rh", "Pd", "Ag", "Cd", "In", "Sn", "Sb", "Te", "I",  "Xe",
    "Cs", "Ba", "La", "Ce", "Pr", "Nd", "Pm", "Sm", "Eu", "Gd", "Tb", "Dy", "Ho", "Er", "Tm", "Yb", "Lu", "Hf",
    "Ta", "W",  "Re", "Os", "Ir", "Pt", "Au", "Hg", "Tl", "Pb", "Bi", "Po", "At", "Rn", "Fr", "Ra", "Ac", "Th",
    "Pa", "U",  "Np", "Pu", "Am", "Cm", "Bk", "Cf", "Es", "Fm", "Md", "No", "Lr", "Rf", "Db", "Sg", "Bh", "Hs",
    "Mt", "Ds", "Rg", "Cn", "Nh", "Fl", "Mc", "Lv", "Ts", "Og"};

struct CudaCancelledError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct CudaUnavailable : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct CudaOutOfMemory : std::runtime_error {
    using std::runtime_error::runtime_error;
};

[[noreturn]] void throw_status(int status) {
    const std::string message = mdsoap_last_error();
    switch (status) {
        case MDSOAP_INVALID_ARGUMENT:
            throw std::invalid_argument(message);
        case MDSOAP_DEVICE_UNAVAILABLE:
            throw CudaUnavailable(message);
        case MDSOAP_OUT_OF_MEMORY:
            throw CudaOutOfMemory(message);
        case MDSOAP_CANCELLED:
            throw CudaCancelledError(message);
        default:
            throw std::runtime_error(message);
    }
}

template <class T>
T option(const py::dict& options, const char* key, T fallback) {
    const py::str name(key);
    if (!options.contains(name) || options[name].is_none()) return fallback;
    return py::cast<T>(options[name]);
}

py::dict child_dict(const py::dict& options, const char* key) {
    const py::str name(key);
    if (!options.contains(name) || options[name].is_none()) return py::dict();
    return py::cast<py::dict>(options[name]);
}

std::vector<double> flat_doubles(const py::dict& d, const char* key) {
    const py::str name(key);
    if (!d.contains(name) || d[name].is_none()) return {};
    auto array = py::array_t<double, py::array::c_style | py::array::forcecast>::ensure(d[name]);
    if (!array) throw std::invalid_argument(std::string("CUDA SOAP payload entry is not numeric: ") + key);
    return std::vector<double>(array.data(), array.data() + array.size());
}

std::vector<int32_t> device_list() {
    // Private selector: the public ExecutionOptions device token cannot carry
    // an index (src/mdescriptor/core/options.py:48-54).
    std::vector<int32_t> ids;
    const char* env = std::getenv("MDSOAP_DEVICES");
    if (!env || !*env) return {0};
    const std::string text(env);
    if (text == "all") {
        const int count = mdsoap_device_count();
        for (int i = 0; i < count; ++i) ids.push_back(i);
        if (ids.empty()) ids.push_back(0);
        return ids;
    }
    size_t start = 0;
    while (start < text.size()) {
        size_t end = text.find(',', start);
        if (end == std::string::npos) end = text.size();
        const std::string token = text.substr(start, end - start);
        if (!token.empty()) ids.push_back((int32_t)std::stoi(token));
        start = end + 1;
    }
    if (ids.empty()) ids.push_back(0);
    return ids;
}

struct CancelContext {
    py::object control;
};

int cancel_probe(void* context) {
    py::gil_scoped_acquire gil;
    auto* ctx = static_cast<CancelContext*>(context);
    try {
        return py::cast<bool>(ctx->control.attr("cancelled")()) ? 1 : 0;
    } catch (py::error_already_set& error) {
        error.discard_as_unraisable("mdsoap cancellation probe");
        return 1;
    }
}

class Backend {
public:
    Backend(std::string name, py::dict options) : name_(std::move(name)), options_(std::move(options)) {
        if (name_ == "NeighborList") {
            // cpp/cuda/src/backend.cu:358-362 option names and defaults.
            list_ = true;
            list_cutoff_ = option(options_, "cutoff", 6.0);
            list_full_ = option(options_, "full_neighbor_list", true);
            list_self_ = option(options_, "self_pairs", false);
            if (!(list_cutoff_ > 0.0) || !std::isfinite(list_cutoff_))
                throw std::invalid_argument("neighbor cutoff must be finite and positive");
            features_ = 4;
            for (const char* label : {"dx", "dy", "dz", "distance"}) labels_.append(label);
            devices_ = device_list();
            return;
        }
        if (name_ == "SphericalExpansion" || name_ == "SoapRadialSpectrum" || name_ == "SoapPowerSpectrum") {
            // cpp/cuda/src/backend.cu:590-602 option names and defaults.
            local_ = true;
            species_ = option(options_, "species", std::vector<int32_t>{});
            local_params_.kind = name_ == "SoapRadialSpectrum"  ? MDSOAP_LOCAL_RADIAL_SPECTRUM
                                 : name_ == "SoapPowerSpectrum" ? MDSOAP_LOCAL_POWER_SPECTRUM
                                                                : MDSOAP_LOCAL_SPHERICAL_EXPANSION;
            local_params_.cutoff = option(options_, "cutoff", 6.0);
            local_params_.density_width = option(options_, "density_width", 0.3);
            local_params_.max_radial = option(options_, "max_radial", 6);
            local_params_.max_angular = option(options_, "max_angular", 4);
            local_params_.n_species = (int32_t)species_.size();
            local_params_.species = species_.data();
            features_ = mdsoap_local_feature_count(&local_params_);
            if (features_ < 0) throw std::invalid_argument(mdsoap_last_error());
            labels_ = labels_option();
            devices_ = device_list();
            return;
        }
        if (name_ != "SOAP")
            throw CudaUnavailable("this CUDA plugin implements SOAP, NeighborList, SphericalExpansion, "
                                  "SoapRadialSpectrum and SoapPowerSpectrum only; '" + name_ +
                                  "' has no CUDA backend here");
        species_ = option(options_, "species", std::vector<int32_t>{});
        if (species_.empty()) throw std::invalid_argument("SOAP species must not be empty");
        n_max_ = option(options_, "n_max", 8);
        l_max_ = option(options_, "l_max", 6);
        r_cut_ = option(options_, "r_cut", 6.0);
        sigma_ = option(options_, "sigma", 1.0);
        if (n_max_ < 1 || n_max_ > 32 || l_max_ < 0 || l_max_ > 20 || r_cut_ <= 0.0 || sigma_ <= 0.0)
            throw std::invalid_argument("invalid CUDA SOAP parameters");
        const std::string rbf = option(options_, "rbf", std::string("gto"));
        if (rbf != "gto" && rbf != "polynomial") throw std::invalid_argument("unsupported CUDA SOAP radial basis");
        polynomial_ = rbf == "polynomial";
        // extended_descriptors_soap.cuh:819-828, 878-884: compression mode and
        // weighting function names.
        const py::dict compression = child_dict(options_, "compression");
        const std::string mode = option(compression, "mode", std::string("off"));
        compression_ = mode == "off" ? MDSOAP_COMPRESSION_OFF
                       : mode == "mu2" ? MDSOAP_COMPRESSION_MU2
                       : mode == "mu1nu1" ? MDSOAP_COMPRESSION_MU1NU1
                       : mode == "crossover" ? MDSOAP_COMPRESSION_CROSSOVER : -1;
        if (compression_ < 0) throw std::invalid_argument("unsupported CUDA SOAP compression");
        const std::string average = option(options_, "average", std::string("inner"));
        if (average != "off" && average != "inner" && average != "outer")
            throw std::invalid_argument("unsupported CUDA SOAP average mode");
        average_ = average == "off" ? MDSOAP_AVERAGE_OFF : average == "inner" ? MDSOAP_AVERAGE_INNER : MDSOAP_AVERAGE_OUTER;
        const py::dict weighting = child_dict(options_, "weighting");
        const std::string function = option(weighting, "function", std::string());
        weighting_function_ = function == "" ? MDSOAP_WEIGHTING_NONE
                              : function == "poly" ? MDSOAP_WEIGHTING_POLY
                              : function == "pow" ? MDSOAP_WEIGHTING_POW
                              : function == "exp" ? MDSOAP_WEIGHTING_EXP : -1;
        if (weighting_function_ < 0) throw std::invalid_argument("unsupported CUDA SOAP weighting");
        // Defaults of SoapKernel._ensure_native (_kernels/core.py:247-254).
        weighting_has_w0_ = weighting.contains("w0");
        weighting_r0_ = option(weighting, "r0", 1.0);
        weighting_c_ = option(weighting, "c", 1.0);
        weighting_d_ = option(weighting, "d", 0.0);
        weighting_m_ = option(weighting, "m", 1.0);
        weighting_w0_ = option(weighting, "w0", 1.0);
        // A species' weight is looked up as an int key, then its decimal
        // string (the adapter's options have been through JSON), then its
        // element symbol; species without an entry weigh 1.0
        // (cpp/cuda/src/extended_descriptors_common.cuh:257-294).
        weights_.assign(species_.size(), 1.0);
        if (compression.contains("species_weighting") && !compression["species_weighting"].is_none()) {
            const py::dict map = py::cast<py::dict>(compression["species_weighting"]);
            for (size_t i = 0; i < species_.size(); ++i) {
                const py::int_ number(species_[i]);
                const py::str text(std::to_string(species_[i]));
                if (map.contains(number)) {
                    weights_[i] = py::cast<double>(map[number]);
                } else if (map.contains(text)) {
                    weights_[i] = py::cast<double>(map[text]);
                } else if (species_[i] >= 1 && species_[i] <= 118) {
                    const py::str symbol(kElementSymbols[species_[i] - 1]);
                    if (map.contains(symbol)) weights_[i] = py::cast<double>(map[symbol]);
                }
            }
        }
        const py::dict output = child_dict(options_, "output");
        const std::string dtype = option(output, "dtype", std::string("float64"));
        if (dtype != "float32" && dtype != "float64") throw std::invalid_argument("CUDA SOAP output dtype must be float32 or float64");
        f64_ = dtype == "float64";
        const py::dict payload = child_dict(options_, "_cuda_payload");
        const py::dict radial = child_dict(payload, "radial_basis");
        const size_t W = (size_t)l_max_ + 1;
        if (polynomial_) {
            // _cuda_payload of the polynomial basis (_kernels/core.py:343-349).
            grid_ = flat_doubles(radial, "radial_grid");
            grid_weights_ = flat_doubles(radial, "radial_weights");
            grid_values_ = flat_doubles(radial, "radial_values");
            if (grid_.size() < 2 || grid_weights_.size() != grid_.size() ||
                grid_values_.size() != (size_t)n_max_ * grid_.size())
                throw std::invalid_argument("CUDA SOAP polynomial payload has an invalid shape");
        } else {
            alphas_ = flat_doubles(radial, "alphas");
            betas_ = flat_doubles(radial, "betas");
            if (alphas_.size() != W * n_max_ || betas_.size() != W * n_max_ * n_max_)
                throw std::invalid_argument("CUDA SOAP GTO payload has an invalid shape");
        }
        mdsoap_params params{};
        params.n_species = (int32_t)species_.size();
        params.species = species_.data();
        params.species_weights = weights_.data();
        params.r_cut = r_cut_;
        params.sigma = sigma_;
        params.n_max = n_max_;
        params.l_max = l_max_;
        params.alphas = alphas_.data();
        params.betas = betas_.data();
        params.radial_basis = polynomial_ ? MDSOAP_RADIAL_POLYNOMIAL : MDSOAP_RADIAL_GTO;
        params.radial_grid_size = (int32_t)grid_.size();
        params.radial_grid = grid_.data();
        params.radial_weights = grid_weights_.data();
        params.radial_values = grid_values_.data();
        params.average = average_;
        params.output_dtype = f64_ ? MDSOAP_FLOAT64 : MDSOAP_FLOAT32;
        params.compression = compression_;
        params.weighting_function = weighting_function_;
        params.weighting_has_w0 = weighting_has_w0_ ? 1 : 0;
        params.weighting_r0 = weighting_r0_;
        params.weighting_c = weighting_c_;
        params.weighting_d = weighting_d_;
        params.weighting_m = weighting_m_;
        params.weighting_w0 = weighting_w0_;
        mdsoap_plan* plan = nullptr;
        const int status = mdsoap_plan_create(&params, &plan);
        if (status != MDSOAP_OK) throw_status(status);
        plan_ = plan;
        features_ = mdsoap_plan_feature_count(plan_);
        const py::str fc_key("_cuda_feature_count");
        if (options_.contains(fc_key) && !options_[fc_key].is_none()) {
            const auto configured = py::cast<int64_t>(options_[fc_key]);
            if (configured > 0 && configured != features_)
                throw std::invalid_argument("CUDA SOAP feature count does not match its layout");
        }
        labels_ = labels_option();
        devices_ = device_list();
    }

    ~Backend() { close(); }

    int64_t feature_count() const { return features_; }

    // Result rows in a recycled page-locked buffer (mdsoap_host_buffer_acquire):
    // the rows arrive by a direct D2H into resident pages, and the buffer goes
    // back to the pool when the array is freed.  Buffers above 1 GiB, or when
    // the host refuses to lock more memory, are ordinary NumPy arrays.
    py::array result_array(int64_t rows) {
        const size_t elem = f64_ ? 8 : 4;
        const size_t bytes = (size_t)rows * (size_t)features_ * elem;
        void* buffer = nullptr;
        if (bytes > 0 && bytes <= ((size_t)1 << 30) && mdsoap_host_buffer_acquire(bytes, &buffer) == MDSOAP_OK) {
            py::capsule owner(buffer, [](void* p) { mdsoap_host_buffer_release(p); });
            const std::vector<py::ssize_t> shape{(py::ssize_t)rows, (py::ssize_t)features_};
            if (f64_) return py::array_t<double>(shape, static_cast<double*>(buffer), owner);
            return py::array_t<float>(shape, static_cast<float*>(buffer), owner);
        }
        if (f64_) return py::array_t<double>({(py::ssize_t)rows, (py::ssize_t)features_});
        return py::array_t<float>({(py::ssize_t)rows, (py::ssize_t)features_});
    }

    py::object compute(py::object batch, py::object control) {
        std::unique_lock<std::mutex> guard(mutex_, std::defer_lock);
        {
            // Never wait for the instance lock while holding the GIL
            // (cpp/cuda/src/backend.cu:339-345).
            py::gil_scoped_release release;
            guard.lock();
        }
        if (closed_ || (plan_ == nullptr && !list_ && !local_)) throw std::runtime_error("CUDA backend is closed");
        auto numbers = py::array_t<int32_t, py::array::c_style | py::array::forcecast>::ensure(batch.attr("numbers"));
        auto positions = py::array_t<double, py::array::c_style | py::array::forcecast>::ensure(batch.attr("positions"));
        auto cells = py::array_t<double, py::array::c_style | py::array::forcecast>::ensure(batch.attr("cells"));
        auto pbc = py::array_t<int32_t, py::array::c_style | py::array::forcecast>::ensure(batch.attr("pbc"));
        auto offsets = py::array_t<int64_t, py::array::c_style | py::array::forcecast>::ensure(batch.attr("offsets"));
        if (!numbers || !positions || !cells || !pbc || !offsets)
            throw std::invalid_argument("structure batch arrays have unsupported types");
        const int64_t structures = (int64_t)offsets.size() - 1;
        if (structures < 0) throw std::invalid_argument("invalid structure batch");
        const int64_t atoms = (int64_t)numbers.size();
        if (positions.size() != 3 * atoms || cells.size() != 9 * structures || pbc.size() != 3 * structures)
            throw std::invalid_argument("structure batch arrays have inconsistent shapes");
        if (!control.is_none()) {
            if (py::hasattr(control, "reset")) control.attr("reset")(structures);
            if (py::cast<bool>(control.attr("cancelled")()))
                throw CudaCancelledError("descriptor computation was cancelled");
        }
        mdsoap_batch view{numbers.data(), positions.data(), cells.data(), pbc.data(), offsets.data(), structures, atoms};
        if (list_) return compute_list(view, structures, control);
        if (local_) return compute_local(view, offsets, structures, control);
        const int64_t rows = average_ == MDSOAP_AVERAGE_OFF ? atoms : structures;
        py::array values = result_array(rows);
        void* out = values.mutable_data();
        CancelContext context{control};
        int status;
        {
            py::gil_scoped_release release;
            status = mdsoap_compute(plan_, &view, rows > 0 ? out : nullptr, devices_.data(), (int32_t)devices_.size(),
                                    control.is_none() ? nullptr : &cancel_probe, &context);
        }
        if (status != MDSOAP_OK) throw_status(status);
        if (!control.is_none() && py::hasattr(control, "mark_completed")) {
            for (int64_t s = 0; s < structures; ++s) control.attr("mark_completed")();
        }
        py::dict result;
        result["values"] = values;
        // The adapter takes an array without its snapshot copy only when the
        // array owns its data (core/result.py:31-50); rows in a recycled
        // page-locked buffer are copied out by the adapter (its block
        // combiner copies every multi-block result anyway), and the buffer
        // goes back to the pool.
        result["_mdescriptor_owned_values"] = values.owndata();
        result["level"] = average_ == MDSOAP_AVERAGE_OFF ? "atom" : "structure";
        if (average_ == MDSOAP_AVERAGE_OFF) {
            py::array_t<int64_t> row_offsets(structures + 1);
            std::copy(offsets.data(), offsets.data() + structures + 1, row_offsets.mutable_data());
            result["row_offsets"] = row_offsets;
        }
        result["labels"] = labels_;
        result["metadata"] = metadata();
        return std::move(result);
    }

    // NeighborList: pair records and features (cpp/cuda/src/backend.cu:418-470).
    py::object compute_list(const mdsoap_batch& view, int64_t structures, py::object control) {
        mdsoap_pairs* pairs = nullptr;
        int status;
        {
            py::gil_scoped_release release;
            status = mdsoap_neighbor_list(&view, list_cutoff_, list_full_ ? 1 : 0, list_self_ ? 1 : 0,
                                          devices_.empty() ? 0 : devices_[0], &pairs);
        }
        if (status != MDSOAP_OK) throw_status(status);
        const int64_t rows = mdsoap_pairs_count(pairs);
        py::array_t<double> values({(py::ssize_t)rows, (py::ssize_t)4});
        py::array_t<double> records({(py::ssize_t)rows, (py::ssize_t)5});
        py::array_t<int64_t> row_offsets(structures + 1);
        mdsoap_pairs_copy(pairs, records.mutable_data(), values.mutable_data(), row_offsets.mutable_data());
        mdsoap_pairs_destroy(pairs);
        if (!control.is_none()) {
            if (py::cast<bool>(control.attr("cancelled")()))
                throw CudaCancelledError("descriptor computation was cancelled");
            if (py::hasattr(control, "mark_completed"))
                for (int64_t s = 0; s < structures; ++s) control.attr("mark_completed")();
        }
        py::dict result;
        result["values"] = values;
        result["_mdescriptor_owned_values"] = true;
        result["level"] = "pair";
        result["row_offsets"] = row_offsets;
        result["pair_records"] = records;
        result["labels"] = labels_;
        result["metadata"] = metadata();
        return std::move(result);
    }

    // Local spectra: float64 atom rows (cpp/cuda/src/backend.cu:590-624).
    py::object compute_local(const mdsoap_batch& view, const py::array_t<int64_t>& offsets, int64_t structures,
                             py::object control) {
        py::array_t<double> values({(py::ssize_t)view.atoms, (py::ssize_t)features_});
        int status;
        {
            py::gil_scoped_release release;
            status = mdsoap_local_compute(&local_params_, &view, values.mutable_data(),
                                          devices_.empty() ? 0 : devices_[0]);
        }
        if (status != MDSOAP_OK) throw_status(status);
        if (!control.is_none()) {
            if (py::cast<bool>(control.attr("cancelled")()))
                throw CudaCancelledError("descriptor computation was cancelled");
            if (py::hasattr(control, "mark_completed"))
                for (int64_t s = 0; s < structures; ++s) control.attr("mark_completed")();
        }
        py::array_t<int64_t> row_offsets(structures + 1);
        std::copy(offsets.data(), offsets.data() + structures + 1, row_offsets.mutable_data());
        py::dict result;
        result["values"] = values;
        result["_mdescriptor_owned_values"] = true;
        result["level"] = "atom";
        result["row_offsets"] = row_offsets;
        result["labels"] = labels_;
        result["metadata"] = metadata();
        return std::move(result);
    }

    py::object predict(py::object, py::object) {
        throw std::invalid_argument("CUDA prediction supports NEP and DPA4C only");
    }

    py::dict metadata() const {
        py::dict result;
        result["descriptor"] = name_;
        result["backend"] = "mdescriptor-cuda";
        py::dict execution;
        execution["device"] = "cuda";
        const py::dict configured = child_dict(options_, "execution");
        execution["num_threads"] = configured.contains("num_threads") ? configured["num_threads"] : py::none();
        result["execution"] = execution;
        return result;
    }

    void close() noexcept {
        std::unique_lock<std::mutex> guard(mutex_, std::defer_lock);
        if (PyGILState_Check()) {
            py::gil_scoped_release release;
            guard.lock();
        } else {
            guard.lock();
        }
        if (!closed_) {
            closed_ = true;
            list_ = false;
            local_ = false;
            if (plan_) mdsoap_plan_destroy(plan_);
            plan_ = nullptr;
        }
    }

private:
    py::list labels_option() const {
        const py::str key("_cuda_labels");
        if (options_.contains(key) && !options_[key].is_none()) {
            py::list configured = py::list(options_[key]);
            if ((int64_t)py::len(configured) == features_) return configured;
        }
        py::list out;
        for (int64_t i = 0; i < features_; ++i) out.append(name_ + ":" + std::to_string(i));
        return out;
    }

    std::string name_;
    py::dict options_;
    std::vector<int32_t> species_;
    std::vector<double> weights_, alphas_, betas_, grid_, grid_weights_, grid_values_;
    bool polynomial_ = false;
    int n_max_ = 8, l_max_ = 6, average_ = MDSOAP_AVERAGE_INNER;
    double r_cut_ = 6.0, sigma_ = 1.0;
    int compression_ = MDSOAP_COMPRESSION_OFF, weighting_function_ = MDSOAP_WEIGHTING_NONE;
    bool weighting_has_w0_ = false;
    double weighting_r0_ = 1.0, weighting_c_ = 1.0, weighting_d_ = 0.0, weighting_m_ = 1.0, weighting_w0_ = 1.0;
    bool f64_ = true;
    bool list_ = false, list_full_ = true, list_self_ = false;  // NeighborList backend
    double list_cutoff_ = 6.0;
    bool local_ = false;  // SphericalExpansion / SoapRadialSpectrum / SoapPowerSpectrum backend
    mdsoap_local_params local_params_{};
    int64_t features_ = 0;
    py::list labels_;
    std::vector<int32_t> devices_;
    mdsoap_plan* plan_ = nullptr;
    bool closed_ = false;
    std::mutex mutex_;
};

}  // namespace

PYBIND11_MODULE(_cuda, module) {
    module.doc() = "MDescriptor CUDA plugin: B200 SOAP engine (mdsoap)";
    module.attr("MODEL_SNAPSHOT_ABI") = 1;
    module.attr("MDSOAP_ABI_VERSION") = mdsoap_abi_version();
    py::register_exception<CudaCancelledError>(module, "CudaCancelledError", PyExc_RuntimeError);
    py::register_exception<CudaUnavailable>(module, "CudaUnavailable", PyExc_ImportError);
    py::register_exception<CudaOutOfMemory>(module, "CudaOutOfMemory", PyExc_MemoryError);

    py::class_<Backend, std::shared_ptr<Backend>>(module, "CudaBackend")
        .def(py::init<std::string, py::dict>())
        .def_property_readonly("feature_count", &Backend::feature_count)
        .def("compute", &Backend::compute, py::arg("batch"), py::arg("control") = py::none())
        .def("predict", &Backend::predict, py::arg("batch"), py::arg("control") = py::none())
        .def("metadata", &Backend::metadata)
        .def("close", &Backend::close);

    module.def("create_backend", [](const std::string& name, const py::dict& options) {
        try {
            return std::make_shared<Backend>(name, options);
        } catch (const CudaUnavailable& error) {
            PyErr_SetString(PyExc_ImportError, error.what());
            throw py::error_already_set();
        } catch (const CudaOutOfMemory& error) {
            PyErr_SetString(PyExc_MemoryError, error.what());
            throw py::error_already_set();
        }
    });
    module.def("create_predictor", [](const std::string&, const py::dict&) -> py::object {
        throw std::invalid_argument("CUDA prediction supports NEP and DPA4C only");
    });
}
