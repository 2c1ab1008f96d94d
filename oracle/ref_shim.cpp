// Test infrastructure only: a C entry layer over the reference's own CPU SOAP
// and neighbour-graph code, compiled from the reference sources in place by
// oracle/build_oracle.py into oracle/_ref/.  Nothing in the product links or
// calls this file.  It is the "reference" CPU baseline that bench.py times and
// the checker that pins the plain-C restatement in oracle/soap_oracle.c.
//
// Wrapped reference entry points:
//   mdescriptor::compute_soap            cpp/src/standalone/soap.cpp:1149
//   mdescriptor::build_neighbor_graph    cpp/src/common/neighbor.cpp:703
//   mdescriptor::compute_neighbor_list   cpp/src/standalone/neighbor_list.cpp:15
#include "mdescriptor/descriptor.hpp"
#include "mdescriptor/local_descriptors.hpp"
#include "mdescriptor/neighbor.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

namespace {
thread_local std::string g_error;

mdescriptor::StructureBatchView make_view(
    const int32_t* numbers, const double* positions, const double* cells,
    const int32_t* pbc, const int64_t* offsets, int64_t structures) {
    mdescriptor::StructureBatchView view;
    view.numbers = numbers;
    view.positions = positions;
    view.cells = cells;
    view.pbc = pbc;
    view.offsets = offsets;
    view.structures = structures;
    view.atoms = offsets[structures];
    return view;
}

struct GraphHandle {
    mdescriptor::NeighborGraph graph;
};
}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_error.c_str(); }

// average: 0 off, 1 inner, 2 outer.  Output is fp64 (rows, features).
int ref_soap_compute(
    const int32_t* numbers, const double* positions, const double* cells,
    const int32_t* pbc, const int64_t* offsets, int64_t structures,
    const int32_t* species, int n_species, double r_cut, int n_max, int l_max,
    double sigma, const double* alphas, const double* betas, int average,
    int num_threads, double* out) {
    try {
        mdescriptor::SoapOptions options;
        options.species.assign(species, species + n_species);
        options.r_cut = r_cut;
        options.n_max = n_max;
        options.l_max = l_max;
        options.sigma = sigma;
        options.radial_basis = 0;
        const size_t count = static_cast<size_t>((l_max + 1) * n_max);
        options.alphas.assign(alphas, alphas + count);
        options.betas.assign(betas, betas + count * n_max);
        options.species_weights.assign(static_cast<size_t>(n_species), 1.0);
        options.compression = 0;
        options.inner_average = average == 1;
        options.outer_average = average == 2;
        options.num_threads = num_threads;
        mdescriptor::compute_soap(
            make_view(numbers, positions, cells, pbc, offsets, structures), options, out, nullptr);
        return 0;
    } catch (const std::exception& error) {
        g_error = error.what();
        return 1;
    }
}

// compute_soap with every SoapOptions field this engine covers: species
// weights (NULL: 1.0 each), compression 0..3, weighting function 0..3 with
// its parameters, w0, and the radial basis (0 GTO: alphas / betas; 1
// polynomial: grid, weights and values [n][grid_size]).
int ref_soap_compute_rbf(
    const int32_t* numbers, const double* positions, const double* cells,
    const int32_t* pbc, const int64_t* offsets, int64_t structures,
    const int32_t* species, int n_species, const double* species_weights, double r_cut, int n_max,
    int l_max, double sigma, const double* alphas, const double* betas, int average, int compression,
    int weighting_function, int weighting_has_w0, double weighting_r0, double weighting_c,
    double weighting_d, double weighting_m, double weighting_w0, int radial_basis, int grid_size,
    const double* grid, const double* grid_weights, const double* grid_values, int num_threads, double* out) {
    try {
        mdescriptor::SoapOptions options;
        options.species.assign(species, species + n_species);
        options.r_cut = r_cut;
        options.n_max = n_max;
        options.l_max = l_max;
        options.sigma = sigma;
        options.radial_basis = radial_basis;
        if (radial_basis == 0) {
            const size_t count = static_cast<size_t>((l_max + 1) * n_max);
            options.alphas.assign(alphas, alphas + count);
            options.betas.assign(betas, betas + count * n_max);
        } else {
            options.radial_grid.assign(grid, grid + grid_size);
            options.radial_weights.assign(grid_weights, grid_weights + grid_size);
            options.radial_values.assign(grid_values, grid_values + static_cast<size_t>(grid_size) * n_max);
        }
        if (species_weights)
            options.species_weights.assign(species_weights, species_weights + n_species);
        else
            options.species_weights.assign(static_cast<size_t>(n_species), 1.0);
        options.compression = compression;
        options.weighting_has_function = weighting_function != 0;
        options.weighting_function = weighting_function;
        options.weighting_has_w0 = weighting_has_w0 != 0;
        options.weighting_r0 = weighting_r0;
        options.weighting_c = weighting_c;
        options.weighting_d = weighting_d;
        options.weighting_m = weighting_m;
        options.weighting_w0 = weighting_w0;
        options.inner_average = average == 1;
        options.outer_average = average == 2;
        options.num_threads = num_threads;
        mdescriptor::compute_soap(
            make_view(numbers, positions, cells, pbc, offsets, structures), options, out, nullptr);
        return 0;
    } catch (const std::exception& error) {
        g_error = error.what();
        return 1;
    }
}

int ref_soap_compute_ex(
    const int32_t* numbers, const double* positions, const double* cells,
    const int32_t* pbc, const int64_t* offsets, int64_t structures,
    const int32_t* species, int n_species, const double* species_weights, double r_cut, int n_max,
    int l_max, double sigma, const double* alphas, const double* betas, int average, int compression,
    int weighting_function, int weighting_has_w0, double weighting_r0, double weighting_c,
    double weighting_d, double weighting_m, double weighting_w0, int num_threads, double* out) {
    return ref_soap_compute_rbf(numbers, positions, cells, pbc, offsets, structures, species, n_species,
                                species_weights, r_cut, n_max, l_max, sigma, alphas, betas, average, compression,
                                weighting_function, weighting_has_w0, weighting_r0, weighting_c, weighting_d,
                                weighting_m, weighting_w0, 0, 0, nullptr, nullptr, nullptr, num_threads, out);
}

struct PairHandle {
    mdescriptor::DescriptorPairTable table;
};

// NeighborList: the reference's pair table (9 columns per row, offsets per structure).
void* ref_neighbor_list(
    const int32_t* numbers, const double* positions, const double* cells,
    const int32_t* pbc, const int64_t* offsets, int64_t structures, double cutoff,
    int full_neighbor_list, int self_pairs, int num_threads) {
    try {
        auto* handle = new PairHandle;
        handle->table = mdescriptor::compute_neighbor_list(
            make_view(numbers, positions, cells, pbc, offsets, structures), cutoff,
            full_neighbor_list != 0, self_pairs != 0, num_threads, nullptr);
        return handle;
    } catch (const std::exception& error) {
        g_error = error.what();
        return nullptr;
    }
}

int64_t ref_neighbor_list_rows(void* handle) {
    return static_cast<int64_t>(static_cast<PairHandle*>(handle)->table.values.size() / 9);
}

void ref_neighbor_list_copy(void* handle, double* values, int64_t* offsets) {
    const auto& table = static_cast<PairHandle*>(handle)->table;
    std::memcpy(values, table.values.data(), table.values.size() * sizeof(double));
    std::memcpy(offsets, table.offsets.data(), table.offsets.size() * sizeof(int64_t));
}

void ref_neighbor_list_free(void* handle) { delete static_cast<PairHandle*>(handle); }

void* ref_graph_build(
    const int32_t* numbers, const double* positions, const double* cells,
    const int32_t* pbc, const int64_t* offsets, int64_t structures, double cutoff,
    int num_threads) {
    try {
        auto* handle = new GraphHandle;
        handle->graph = mdescriptor::build_neighbor_graph(
            make_view(numbers, positions, cells, pbc, offsets, structures), cutoff, nullptr,
            num_threads);
        return handle;
    } catch (const std::exception& error) {
        g_error = error.what();
        return nullptr;
    }
}

int64_t ref_graph_pairs(void* handle) {
    return static_cast<int64_t>(static_cast<GraphHandle*>(handle)->graph.atoms_data().size());
}

void ref_graph_copy(
    void* handle, int64_t* offsets, int32_t* atoms, int32_t* shifts, double* displacements,
    double* distance2) {
    const auto& graph = static_cast<GraphHandle*>(handle)->graph;
    std::memcpy(offsets, graph.offsets().data(), graph.offsets().size() * sizeof(int64_t));
    std::memcpy(atoms, graph.atoms_data().data(), graph.atoms_data().size() * sizeof(int32_t));
    std::memcpy(shifts, graph.shifts().data(), graph.shifts().size() * sizeof(int32_t));
    std::memcpy(displacements, graph.displacements().data(),
                graph.displacements().size() * sizeof(double));
    std::memcpy(distance2, graph.distance2().data(), graph.distance2().size() * sizeof(double));
}

void ref_graph_free(void* handle) { delete static_cast<GraphHandle*>(handle); }

}  // extern "C"
