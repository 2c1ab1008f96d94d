// mdsoap: host side of the B200 SOAP engine and its C ABI (include/mdsoap.h).
//
// One plan = one SOAP configuration.  Device state (constants, workspaces,
// streams, pinned staging) is created lazily per device on the first compute
// there, so building a plan touches no GPU (the reference's construction-time
// contract, tests/test_cuda_backend.py:266-279).
#include "../../include/mdsoap.h"
#include "launchers.cuh"
#include "neighbor_list.cuh"
#include "csr.cuh"
#include "local_spectra.cuh"

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <unordered_map>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

using namespace mdsoap;

namespace {

thread_local std::string g_error;

int fail(int status, const std::string& message) {
    g_error = message;
    return status;
}

struct Failure {
    int status;
    std::string message;
};

[[noreturn]] void raise(int status, const std::string& message) { throw Failure{status, message}; }

void check(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return;
    const std::string text = std::string(what) + ": " + cudaGetErrorString(err);
    if (err == cudaErrorMemoryAllocation) raise(MDSOAP_OUT_OF_MEMORY, text);
    if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver || err == cudaErrorInvalidDevice ||
        err == cudaErrorDevicesUnavailable || err == cudaErrorInitializationError)
        raise(MDSOAP_DEVICE_UNAVAILABLE, text);
    raise(MDSOAP_INTERNAL, text);
}

std::string device_error_text(unsigned bits) {
    if (bits & kErrUnknownSpecies) return "batch contains an atomic number outside calculator species";
    if (bits & kErrMixedPbc) return "mixed periodicity is not supported; use all-zero or all-one pbc";
    if (bits & kErrSingularCell) return "cells must be nonsingular";
    if (bits & kErrWrapRange) return "periodic image range exceeds integer range";
    if (bits & kErrPairCapacity) return "neighbour list: a centre has more pairs than the GPU list holds (2048)";
    if (bits & kErrExtendedRange) return "neighbor extended atom index exceeds int32 range";
    if (bits & kErrTailTimeout) return "tail kernel: a coefficient block copy did not complete in time";
    if (bits & kErrLocalSeries) return "local descriptor radial integral overflow";
    return "device error";
}

// Injected allocation failure, for the out-of-memory tests: with
// MDSOAP_TEST_FAIL_ALLOC=<bytes> set, every engine device allocation of at
// least that many bytes returns cudaErrorMemoryAllocation without calling
// cudaMalloc, so the OUT_OF_MEMORY path (status, plugin exception, adapter
// error code) is exercised on the host, with no real exhaustion of a GPU.
cudaError_t engine_malloc(void** ptr, size_t bytes) {
    if (const char* env = std::getenv("MDSOAP_TEST_FAIL_ALLOC")) {
        const long long limit = std::atoll(env);
        if (limit > 0 && bytes >= (size_t)limit) {
            *ptr = nullptr;
            return cudaErrorMemoryAllocation;
        }
    }
    return cudaMalloc(ptr, bytes);
}

// Host-side NVTX range (upload, binning, expansion, tail, D2H), closed at scope exit.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

// Grow-only device buffer.
struct DeviceBytes {
    void* ptr = nullptr;
    size_t size = 0;
    void reserve(size_t bytes, const char* what) {
        if (bytes <= size) return;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        size = 0;
        const size_t rounded = std::max<size_t>(bytes + bytes / 8, 256);
        check(engine_malloc(&ptr, rounded), what);
        size = rounded;
    }
    template <class T>
    T* as() const { return static_cast<T*>(ptr); }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        size = 0;
    }
};

struct PinnedBytes {
    void* ptr = nullptr;
    size_t size = 0;
    void reserve(size_t bytes) {
        if (bytes <= size) return;
        if (ptr) cudaFreeHost(ptr);
        ptr = nullptr;
        size = 0;
        check(cudaMallocHost(&ptr, bytes), "pinned staging allocation");
        size = bytes;
    }
    void release() {
        if (ptr) cudaFreeHost(ptr);
        ptr = nullptr;
        size = 0;
    }
};

// Device workspace for one batch (or one shard of one).
struct Workspace {
    DeviceBytes numbers, positions, cells, pbc, offsets;
    DeviceBytes info, struct_of, type, bin_of, wrap, sorted, bin_start, bin_cursor, spos;
    DeviceBytes cbuf, pbuf, rbuf;
    DeviceBytes edges, edge_info, edge_count;  // edge-list split: per-centre edge slots of a chunk
    void release() {
        for (DeviceBytes* b : {&numbers, &positions, &cells, &pbc, &offsets, &info, &struct_of, &type, &bin_of,
                               &wrap, &sorted, &bin_start, &bin_cursor, &spos, &cbuf, &pbuf, &rbuf, &edges,
                               &edge_info, &edge_count})
            b->release();
    }
    BinView bins(unsigned* error) {
        BinView v;
        v.info = info.as<StructInfo>();
        v.struct_of = struct_of.as<int32_t>();
        v.type = type.as<int32_t>();
        v.bin_of = bin_of.as<int32_t>();
        v.wrap = wrap.as<int32_t>();
        v.sorted = sorted.as<int32_t>();
        v.bin_start = bin_start.as<int32_t>();
        v.bin_cursor = bin_cursor.as<int32_t>();
        v.error = error;
        v.spos = spos.as<double4>();
        return v;
    }
    void reserve_bins(int64_t atoms, int64_t structures) {
        const size_t a = (size_t)std::max<int64_t>(atoms, 1);
        info.reserve(sizeof(StructInfo) * (size_t)std::max<int64_t>(structures, 1), "bin info");
        struct_of.reserve(4 * a, "bin struct_of");
        type.reserve(4 * a, "bin type");
        bin_of.reserve(4 * a, "bin bin_of");
        wrap.reserve(12 * a, "bin wrap");
        sorted.reserve(4 * a, "bin sorted");
        spos.reserve(32 * a, "bin sorted positions");
        const size_t bins = (size_t)(2 * atoms + 8 * structures + 8);
        bin_start.reserve(4 * bins, "bin starts");
        bin_cursor.reserve(4 * bins, "bin cursors");
    }
};

using launch::CenterLauncher;
using launch::StructureLauncher;

// Kernel variants.  Slot lengths bound 2l+1 of the channels a lane owns per
// pass: channels are sorted by l descending, 32 per slot, and with n_max <= 8
// the channels ranked 32s.. have l <= l_max - 4s.  Within a (n, l) class the
// variants trade species register banks (MAXT, fewer passes) against
// registers per thread (MINB resident CTAs per SM).
struct Variant {
    int cls, maxt, l0, l1, l2, nmax, lmax, minb;
    CenterLauncher center;
    const void* (*center_sym)();
    StructureLauncher structure;
    const void* (*structure_sym)();
    bool paired = false;   // paired-channel kernel (soap_paired_kernel), l_max == lmax exactly
    bool precise = false;  // paired: full-accuracy radial factors (float64 rows)
    const char* name = "";  // kernel and template arguments, for measurement records
    CenterLauncher tail = nullptr;        // paired: soap_tail_kernel<lmax, maxt>
    const void* (*tail_sym)() = nullptr;
    const void* (*split_sym)() = nullptr; // paired: the expansion kernel without tail code
    CenterLauncher tail_generic = nullptr;  // paired: soap_tail_generic_kernel<lmax>
    const void* (*tail_generic_sym)() = nullptr;
    CenterLauncher walk = nullptr;          // paired: walk-only kernel (edge-list split)
    const void* (*walk_sym)() = nullptr;
    CenterLauncher expand = nullptr;        // paired: expansion-only kernel (edge-list split)
    const void* (*expand_sym)() = nullptr;
};

#define MDSOAP_VARIANT(CLS, T, A, B, C, N, L, MB)                                                           \
    Variant {                                                                                                \
        CLS, T, A, B, C, N, L, MB, &launch::center<T, A, B, C, N, L, MB>,                                    \
            &launch::center_symbol<T, A, B, C, N, L, MB>, &launch::structure<L>, &launch::structure_symbol<L>, \
            false, false, "soap_center_kernel<" #T ", " #A ", " #B ", " #C ", " #N ", " #L ", " #MB ">"        \
    }

// First entry of each class is the default (chosen by measurement on B200,
// config shapes 1-5); the other member trades species register banks against
// resident CTAs (MDSOAP_VARIANT=k).
const Variant kVariants[] = {
    MDSOAP_VARIANT(0, 4, 7, 0, 0, 8, 3, 3),         // n <= 8, l <= 3
    MDSOAP_VARIANT(0, 8, 7, 0, 0, 8, 3, 2),
    MDSOAP_VARIANT(1, 3, 9, 1, 0, 8, 4, 3),         // n <= 8, l == 4
    MDSOAP_VARIANT(1, 6, 9, 1, 0, 8, 4, 2),
    MDSOAP_VARIANT(2, 4, 13, 5, 0, 8, 6, 2),        // n <= 8, l in 5..6
    MDSOAP_VARIANT(3, 2, 17, 9, 1, 8, 8, 2),        // n <= 8, l in 7..8
    MDSOAP_VARIANT(4, 1, 41, 0, 0, 32, 20, 1),  // any n <= 32, l <= 20
};

#define MDSOAP_PAIRED_VARIANT(T, L, PREC, MB)                                                                \
    Variant {                                                                                                \
        -1, T, 0, 0, 0, 8, L, MB, &launch::paired<T, L, PREC, MB>, &launch::paired_symbol<T, L, PREC, MB>,   \
            &launch::structure<L>, &launch::structure_symbol<L>, true, PREC,                                 \
            "soap_paired_kernel<" #T ", " #L ", " #PREC ", " #MB ">", &launch::tail<L, T>,                   \
            &launch::tail_symbol<L, T>, &launch::paired_split_symbol<T, L, PREC, MB>,                        \
            &launch::tail_generic<L>, &launch::tail_generic_symbol<L>, &launch::paired_walk<PREC>,           \
            &launch::paired_walk_symbol<PREC>, &launch::paired_expand<(PREC ? 2 : 1), L, PREC, 3>,          \
            &launch::paired_expand_symbol<(PREC ? 2 : 1), L, PREC, 3>                                        \
    }

// Paired-channel kernels: the default wherever they apply (n_max <= 8,
// n_max (1 + (l_max + 1) / 2) <= 32 lanes, an instantiated l_max, and radial
// factors that stay normal doubles; see paired_applies).
const Variant kPairedVariants[] = {
    MDSOAP_PAIRED_VARIANT(4, 0, false, 2), MDSOAP_PAIRED_VARIANT(4, 0, true, 2),
    MDSOAP_PAIRED_VARIANT(4, 1, false, 2), MDSOAP_PAIRED_VARIANT(4, 1, true, 2),
    MDSOAP_PAIRED_VARIANT(4, 2, false, 2), MDSOAP_PAIRED_VARIANT(4, 2, true, 2),
    MDSOAP_PAIRED_VARIANT(4, 3, false, 2), MDSOAP_PAIRED_VARIANT(4, 3, true, 2),
    MDSOAP_PAIRED_VARIANT(4, 4, false, 2), MDSOAP_PAIRED_VARIANT(4, 4, true, 2),
    MDSOAP_PAIRED_VARIANT(4, 5, false, 2), MDSOAP_PAIRED_VARIANT(4, 5, true, 2),
    MDSOAP_PAIRED_VARIANT(4, 6, false, 2), MDSOAP_PAIRED_VARIANT(4, 6, true, 2),
    // Fewer register banks for plans with fewer species (fewer registers).
    MDSOAP_PAIRED_VARIANT(3, 6, false, 2), MDSOAP_PAIRED_VARIANT(3, 6, true, 2),
};

#define MDSOAP_POLY_VARIANT(T, L)                                                                            \
    Variant {                                                                                                \
        -1, T, 0, 0, 0, 8, L, 2, &launch::poly<T, L>, &launch::poly_symbol<T, L>, &launch::structure<L>,     \
            &launch::structure_symbol<L>, true, true, "soap_paired_kernel<" #T ", " #L ", true, 2, false, true>" \
    }

// Polynomial radial basis kernels (same applicability as the paired kernels).
const Variant kPolyVariants[] = {
    MDSOAP_POLY_VARIANT(4, 0), MDSOAP_POLY_VARIANT(4, 1), MDSOAP_POLY_VARIANT(4, 2), MDSOAP_POLY_VARIANT(4, 3),
    MDSOAP_POLY_VARIANT(4, 4), MDSOAP_POLY_VARIANT(4, 5), MDSOAP_POLY_VARIANT(4, 6),
};

const Variant* poly_variant(int n_max, int l_max) {
    if (n_max > 8 || n_max * (1 + (l_max + 1) / 2) > 32) return nullptr;
    for (const Variant& v : kPolyVariants)
        if (v.lmax == l_max) return &v;
    return nullptr;
}

// The paired kernel for (n_max, l_max) with the fewest species register banks
// that still hold all `species` of the coefficient block in one pass (the
// four-bank kernel, in several passes, beyond that).
const Variant* paired_variant(int n_max, int l_max, bool precise, int species) {
    if (n_max > 8 || n_max * (1 + (l_max + 1) / 2) > 32) return nullptr;
    const Variant* best = nullptr;
    for (const Variant& v : kPairedVariants) {
        if (v.lmax != l_max || v.precise != precise) continue;
        const bool fits = v.maxt >= species;
        if (!best) best = &v;
        else if (fits && (best->maxt < species || v.maxt < best->maxt)) best = &v;
        else if (!fits && best->maxt < species && v.maxt > best->maxt) best = &v;
    }
    return best;
}

int variant_class(int n_max, int l_max) {
    if (n_max <= 8) {
        if (l_max <= 3) return 0;
        if (l_max == 4) return 1;
        if (l_max <= 6) return 2;
        if (l_max <= 8) return 3;
    }
    return 4;
}

// The want-th member of the class of (n_max, l_max), or its first member
// when `want` is out of range.
const Variant& pick_variant(int n_max, int l_max, int want) {
    const int cls = variant_class(n_max, l_max);
    const Variant* first = nullptr;
    int k = 0;
    for (const Variant& v : kVariants) {
        if (v.cls != cls) continue;
        if (!first) first = &v;
        if (k++ == want) return v;
    }
    return *first;
}

// fp64 FMA throughput probe: kProbeChains independent dependent-FMA chains per
// thread, all in registers, result kept live through a store.
constexpr int kProbeChains = 8;
__global__ void fma_probe_kernel(double* sink, int iters) {
    double v[kProbeChains];
    const double a = 1.0 + 1e-9 * threadIdx.x, b = 1e-12;
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) v[c] = 0.5 + c;
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int c = 0; c < kProbeChains; ++c) v[c] = fma(v[c], a, b);
    }
    double s = 0.0;
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) s += v[c];
    sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// The engine's exp() (expneg.cuh) beside CUDA's exp() on the same arguments.
__global__ void exp_probe_kernel(const double* __restrict__ x, int64_t count, double* __restrict__ ours,
                                 double* __restrict__ cuda_exp) {
    __shared__ double table[32];
    if (threadIdx.x < 32) table[threadIdx.x] = kExp2Table[threadIdx.x];
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        ours[i] = exp_nonpositive(x[i], table);
        cuda_exp[i] = exp(x[i]);
    }
}

// The radial-factor forms the kernels use, beside pref * CUDA's exp() of the
// same argument: 0 scaled_exp<true> (float64 rows), 1 scaled_exp<false>
// (float32 rows, one-kernel walk), 2 scaled_exp_folded<64> (float32 rows,
// expansion-only kernel).
__global__ void radial_probe_kernel(int form, const double* __restrict__ u, const double* __restrict__ e,
                                    const double* __restrict__ pref, int64_t count, double* __restrict__ ours,
                                    double* __restrict__ cuda_exp) {
    __shared__ double t32[32], t64[64];
    for (int i = threadIdx.x; i < 64; i += blockDim.x) {
        t64[i] = kExp2Table64[i];
        if (i < 32) t32[i] = kExp2Table[i];
    }
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        const double x = -e[i] * u[i];
        double v;
        if (form == 0)
            v = scaled_exp<true>(x, pref[i], t32);
        else if (form == 1)
            v = scaled_exp<false>(x, pref[i], t32);
        else
            v = scaled_exp_folded<64>(u[i], -e[i] * folded_scale(64), pref[i], t64);
        ours[i] = v;
        cuda_exp[i] = pref[i] * exp(x);
    }
}

// The tail kernel's bounded wait made to run out: one thread arms an mbarrier
// for 16 bytes of copies and issues none, so the phase cannot complete; the
// wait (bulk::wait, the tail kernel's own) gives up after limit_ns and the
// kernel sets kErrTailTimeout, exactly as the tail kernel does.  No copy is
// ever in flight, so the shared memory is free when the CTA exits.
__global__ void bounded_wait_probe_kernel(unsigned* error, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        bulk::barrier_init(&bar, 1);
        bulk::barrier_init_fence();
        bulk::arrive_expect(&bar, 16u);
        if (!bulk::wait(&bar, 0u, limit_ns)) atomicOr(error, kErrTailTimeout);
    }
}

}  // namespace

// ---------------------------------------------------------------------------

struct DeviceState {
    int device = -1;
    cudaStream_t compute = nullptr;
    cudaStream_t copy = nullptr;
    cudaEvent_t computed[2] = {nullptr, nullptr};
    cudaEvent_t copied[2] = {nullptr, nullptr};
    DeviceBytes items, betas, species, error, poly;
    Workspace work;
    DeviceBytes out[2];
    PinnedBytes staging[2];
    bool smem_configured = false;
    int64_t tail_grid = 0;    // persistent tail kernel: resident CTAs on this device
    int64_t center_grid = 0;  // paired kernel: resident CTAs on this device (0: one CTA per kWarps centres)
    int64_t walk_grid = 0;    // edge-list split: resident CTAs of the walk-only kernel
    int64_t expand_grid = 0;  // edge-list split: resident CTAs of the expansion-only kernel
    cudaEvent_t timing[4] = {nullptr, nullptr, nullptr, nullptr};  // bin | centre | tail | structure
    bool timed = false;  // the last device call recorded the timing events
    // Split-tail plans: per chunk of centres, an event after its expansion
    // launch and one after its tail launch (the timed call used the first
    // split_marks of them).
    std::vector<cudaEvent_t> marks;
    size_t split_marks = 0;
    std::mutex mutex;

    ~DeviceState() {
        if (device < 0) return;
        int previous = 0;
        cudaGetDevice(&previous);
        cudaSetDevice(device);
        if (compute) cudaStreamSynchronize(compute);
        if (copy) cudaStreamSynchronize(copy);
        work.release();
        for (auto& b : out) b.release();
        for (auto& b : staging) b.release();
        items.release();
        betas.release();
        species.release();
        error.release();
        for (auto& e : computed)
            if (e) cudaEventDestroy(e);
        for (auto& e : copied)
            if (e) cudaEventDestroy(e);
        for (auto& e : timing)
            if (e) cudaEventDestroy(e);
        for (auto& e : marks)
            if (e) cudaEventDestroy(e);
        if (compute) cudaStreamDestroy(compute);
        if (copy) cudaStreamDestroy(copy);
        cudaSetDevice(previous);
    }
};

struct mdsoap_plan {
    int n_species = 0, n_max = 0, l_max = 0, average = 0, out_dtype = 0, compression = 0;
    double r_cut = 0, sigma = 0, cutoff = 0;
    std::vector<int32_t> species;
    std::vector<double> weights, alphas, betas;
    std::vector<double> poly;  // polynomial basis: nodes [Q], weighted values [Q][n_max]
    std::vector<RadialItem> items;
    SoapTables tab{};
    const Variant* variant = nullptr;
    size_t center_smem = 0;
    size_t structure_smem = 0;
    size_t tail_smem = 0;      // split tail kernel (tab.split_tail)
    size_t walk_smem = 0;      // edge-list split: walk-only kernel (tab.edge_cap > 0)
    CenterLauncher walk_launch = nullptr;   // its launcher and symbol (paired or centre plans)
    const void* (*walk_symbol)() = nullptr;
    int64_t edge_chunk = 1 << 30;  // centre plans: centres per walk / centre-kernel pair of launches
    size_t expand_smem = 0;    // edge-list split: expansion-only kernel
    int32_t expand_chunk = 0;       // its edge chunk and per-warp shared memory (one species per pass,
    int32_t expand_warp_bytes = 0;  // raw sums flushed straight to the tail's global scratch)
    CenterLauncher expand_launch = nullptr;
    const void* (*expand_symbol)() = nullptr;
    std::string kernel_label;  // the kernel(s) a step launches after binning
    int64_t tail_chunk = 1 << 30; // centres per expansion / tail pair of launches (MDSOAP_TAIL_CHUNK)
    int64_t csize = 0;
    int64_t features = 0;
    bool timing = false;
    std::atomic<int64_t> launches{0};  // kernels this plan has launched, all devices
    std::mutex devices_mutex;
    std::vector<std::unique_ptr<DeviceState>> devices;

    size_t out_elem() const { return out_dtype == MDSOAP_FLOAT64 ? 8 : 4; }

    DeviceState& state(int device);
    void configure_smem(DeviceState& st);
    void bin(DeviceState& st, const DeviceBatch& b, cudaStream_t stream, unsigned* error);
    void run_block(DeviceState& st, const DeviceBatch& b, int64_t s0, int64_t s1, int64_t a0, int64_t a1,
                   void* out, cudaStream_t stream, unsigned* error, cudaEvent_t after_center = nullptr,
                   bool mark_chunks = false);
    void shard_compute(int device, const mdsoap_batch& batch, int64_t s0, int64_t s1, char* out,
                       mdsoap_cancel_fn cancel, void* ctx, std::atomic<bool>& stop);
};

DeviceState& mdsoap_plan::state(int device) {
    std::lock_guard<std::mutex> lock(devices_mutex);
    for (auto& st : devices)
        if (st->device == device) return *st;
    int count = 0;
    const cudaError_t probe = cudaGetDeviceCount(&count);
    if (probe != cudaSuccess || count == 0)
        raise(MDSOAP_DEVICE_UNAVAILABLE,
              std::string("no CUDA device available: ") + cudaGetErrorString(probe));
    if (device < 0 || device >= count) raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device index out of range");
    auto st = std::make_unique<DeviceState>();
    check(cudaSetDevice(device), "cudaSetDevice");
    st->device = device;
    check(cudaStreamCreateWithFlags(&st->compute, cudaStreamNonBlocking), "stream");
    check(cudaStreamCreateWithFlags(&st->copy, cudaStreamNonBlocking), "stream");
    for (int i = 0; i < 2; ++i) {
        check(cudaEventCreateWithFlags(&st->computed[i], cudaEventDisableTiming), "event");
        check(cudaEventCreateWithFlags(&st->copied[i], cudaEventDisableTiming), "event");
    }
    st->items.reserve(sizeof(RadialItem) * items.size(), "radial items");
    check(cudaMemcpy(st->items.ptr, items.data(), sizeof(RadialItem) * items.size(), cudaMemcpyHostToDevice),
          "upload radial items");
    st->betas.reserve(8 * betas.size(), "betas");
    check(cudaMemcpy(st->betas.ptr, betas.data(), 8 * betas.size(), cudaMemcpyHostToDevice), "upload betas");
    st->species.reserve(4 * species.size(), "species");
    check(cudaMemcpy(st->species.ptr, species.data(), 4 * species.size(), cudaMemcpyHostToDevice), "upload species");
    if (!poly.empty()) {
        st->poly.reserve(8 * poly.size(), "polynomial basis");
        check(cudaMemcpy(st->poly.ptr, poly.data(), 8 * poly.size(), cudaMemcpyHostToDevice), "upload polynomial basis");
    }
    st->error.reserve(64, "error word");
    check(cudaMemset(st->error.ptr, 0, 64), "clear error word");
    configure_smem(*st);
    devices.push_back(std::move(st));
    return *devices.back();
}

void mdsoap_plan::configure_smem(DeviceState& st) {
    int optin = 0;
    check(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, st.device), "smem attribute");
    if (center_smem > (size_t)optin || structure_smem > (size_t)optin)
        raise(MDSOAP_INVALID_ARGUMENT, "SOAP parameters need more shared memory than the device offers");
    // The attribute is a per-kernel ceiling shared by every plan using the same
    // instantiation, so raise it to the device maximum rather than this plan's need.
    check(cudaFuncSetAttribute(variant->center_sym(), cudaFuncAttributeMaxDynamicSharedMemorySize, optin),
          "center kernel smem");
    check(cudaFuncSetAttribute(variant->structure_sym(), cudaFuncAttributeMaxDynamicSharedMemorySize, optin),
          "structure kernel smem");
    if (variant->tail_sym) {
        // The tail kernels' static shared memory (the mbarriers): the dynamic
        // ceiling is what remains of the opt-in maximum.
        for (const void* sym : {variant->tail_sym(), variant->tail_generic_sym()}) {
            cudaFuncAttributes attr{};
            check(cudaFuncGetAttributes(&attr, sym), "tail kernel attributes");
            check(cudaFuncSetAttribute(sym, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       optin - (int)attr.sharedSizeBytes),
                  "tail kernel smem");
        }
        if (tab.split_tail) {
            int per_sm = 0, sms = 0;
            const void* sym = tab.split_tail == 2 ? variant->tail_generic_sym() : variant->tail_sym();
            check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sym, kWarps * 32, tail_smem),
                  "tail kernel occupancy");
            check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, st.device), "SM count");
            st.tail_grid = (int64_t)std::max(per_sm, 1) * sms;
        }
    }
    if (variant->split_sym)
        check(cudaFuncSetAttribute(variant->split_sym(), cudaFuncAttributeMaxDynamicSharedMemorySize, optin),
              "centre kernel smem");
    if (tab.edge_cap > 0) {
        int per_sm = 0, sms = 0;
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, st.device), "SM count");
        check(cudaFuncSetAttribute(walk_symbol(), cudaFuncAttributeMaxDynamicSharedMemorySize, optin),
              "walk kernel smem");
        check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, walk_symbol(), kWarps * 32, walk_smem),
              "walk kernel occupancy");
        st.walk_grid = (int64_t)std::max(per_sm, 1) * sms;
        if (expand_symbol) {
            check(cudaFuncSetAttribute(expand_symbol(), cudaFuncAttributeMaxDynamicSharedMemorySize, optin),
                  "expansion kernel smem");
            check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, expand_symbol(), kWarps * 32, expand_smem),
                  "expansion kernel occupancy");
            st.expand_grid = (int64_t)std::max(per_sm, 1) * sms;
        }
    }
    // The paired kernel runs persistent: as many CTAs as fit on the device,
    // each over a contiguous range of centres.  MDSOAP_PERSISTENT=0 launches
    // one CTA per kWarps centres instead (measurement knob).
    const char* persistent_env = std::getenv("MDSOAP_PERSISTENT");
    if (variant->paired && !(persistent_env && persistent_env[0] == '0')) {
        const void* sym = (tab.split_tail && variant->split_sym) ? variant->split_sym() : variant->center_sym();
        int per_sm = 0, sms = 0;
        check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sym, kWarps * 32, center_smem),
              "centre kernel occupancy");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, st.device), "SM count");
        st.center_grid = (int64_t)std::max(per_sm, 1) * sms;
    }
    st.smem_configured = true;
}

void mdsoap_plan::bin(DeviceState& st, const DeviceBatch& b, cudaStream_t stream, unsigned* error) {
    if (b.structures == 0) return;
    NvtxRange range("mdsoap bin");
    st.work.reserve_bins(b.atoms, b.structures);
    bin_structures_kernel<<<(unsigned)b.structures, 256, 0, stream>>>(b, st.work.bins(error), cutoff,
                                                                       st.species.as<int32_t>(), n_species);
    check(cudaGetLastError(), "bin kernel launch");
    launches.fetch_add(1, std::memory_order_relaxed);
}

// Centres [a0, a1) = atoms of structures [s0, s1); rows go to `out` starting
// at the block's first row.
void mdsoap_plan::run_block(DeviceState& st, const DeviceBatch& b, int64_t s0, int64_t s1, int64_t a0, int64_t a1,
                            void* out, cudaStream_t stream, unsigned* error, cudaEvent_t after_center,
                            bool mark_chunks) {
    const int64_t centers = a1 - a0;
    const int64_t csize = tab.csize;
    SoapPointers p{};
    p.positions = b.positions;
    p.bins = st.work.bins(error);
    p.items = st.items.as<RadialItem>();
    p.betas = st.betas.as<double>();
    p.poly = st.poly.as<double>();
    p.out = out;
    p.out_row_begin = a0;
    p.center_begin = a0;
    p.center_end = a1;
    if (average == MDSOAP_AVERAGE_INNER) {
        st.work.cbuf.reserve(8 * (size_t)std::max<int64_t>(centers, 1) * csize, "inner-average scratch");
        p.cbuf = st.work.cbuf.as<double>();
    } else if (average == MDSOAP_AVERAGE_OUTER) {
        st.work.pbuf.reserve(8 * (size_t)std::max<int64_t>(centers, 1) * features, "outer-average scratch");
        p.pbuf = st.work.pbuf.as<double>();
    }
    p.grid_begin = a0;
    p.grid_end = a1;
    if (tab.split_tail) {
        // Expansion kernel, then tail kernel (soap_tail_kernel) on the raw-sum
        // blocks it left in scratch; MDSOAP_TAIL_CHUNK alternates the two over
        // chunks of centres instead (smaller scratch; measured slower on
        // config 2, where one pair of launches is fastest).
        const int64_t chunk = std::min<int64_t>(centers, tail_chunk);
        st.work.rbuf.reserve(8 * (size_t)std::max<int64_t>(chunk, 1) * tab.rsize, "coefficient scratch");
        p.rbuf = st.work.rbuf.as<double>();
        st.split_marks = 0;
        // Timing: an event after each expansion launch and after each tail launch.
        auto mark = [&]() {
            if (!mark_chunks) return;
            if (st.split_marks == st.marks.size()) {
                cudaEvent_t e = nullptr;
                check(cudaEventCreate(&e), "timing event");
                st.marks.push_back(e);
            }
            check(cudaEventRecord(st.marks[st.split_marks++], stream), "timing event");
        };
        const bool edge_lists = tab.edge_cap > 0;
        if (edge_lists) {
            const size_t slots = (size_t)std::max<int64_t>(chunk, 1);
            st.work.edges.reserve(slots * (size_t)tab.edge_cap * sizeof(double4), "edge slots");
            st.work.edge_info.reserve(slots * (size_t)tab.edge_cap * sizeof(int32_t), "edge slots");
            st.work.edge_count.reserve(slots * sizeof(int32_t), "edge counts");
            p.edges = st.work.edges.as<double4>();
            p.edge_info = st.work.edge_info.as<int32_t>();
            p.edge_count = st.work.edge_count.as<int32_t>();
        }
        for (int64_t c0 = a0; c0 < a1; c0 += chunk) {
            p.grid_begin = c0;
            p.grid_end = std::min(a1, c0 + chunk);
            const int64_t one_per_warp = (p.grid_end - c0 + kWarps - 1) / kWarps;
            int64_t grid = one_per_warp;
            if (st.center_grid > 0) grid = std::min(grid, st.center_grid);
            if (edge_lists) {
                // Walk (edges to the slots), expansion from the slots, then
                // the fused kernel over the centres whose slot overflowed.
                NvtxRange range("mdsoap walk + expansion");
                SoapTables walk_tab = tab;
                walk_tab.warp_bytes = paired::kHeaderBytes;
                variant->walk(dim3((unsigned)std::min(one_per_warp, std::max<int64_t>(st.walk_grid, 1))), walk_smem,
                              stream, walk_tab, p);
                check(cudaGetLastError(), "walk kernel launch");
                SoapTables et = tab;
                et.chunk = expand_chunk;
                et.r_global = 1;
                et.warp_bytes = expand_warp_bytes;
                et.r_offset = 0;
                expand_launch(dim3((unsigned)std::min(one_per_warp, std::max<int64_t>(st.expand_grid, 1))),
                              expand_smem, stream, et, p);
                check(cudaGetLastError(), "expansion kernel launch");
                variant->center(dim3((unsigned)grid), center_smem, stream, tab, p);
                check(cudaGetLastError(), "centre kernel launch");
                launches.fetch_add(2, std::memory_order_relaxed);
            } else {
                NvtxRange range("mdsoap expansion");
                variant->center(dim3((unsigned)grid), center_smem, stream, tab, p);
                check(cudaGetLastError(), "centre kernel launch");
            }
            mark();
            // Persistent tail: the resident CTAs stride over the block's centres.
            const int64_t tail_ctas = std::min<int64_t>(p.grid_end - c0, std::max<int64_t>(st.tail_grid, 1));
            NvtxRange range("mdsoap tail");
            (tab.split_tail == 2 ? variant->tail_generic : variant->tail)(dim3((unsigned)tail_ctas), tail_smem,
                                                                          stream, tab, p);
            check(cudaGetLastError(), "tail kernel launch");
            mark();
            launches.fetch_add(2, std::memory_order_relaxed);
        }
        p.grid_begin = a0;
        p.grid_end = a1;
        p.edges = nullptr;
        p.edge_info = nullptr;
        p.edge_count = nullptr;
    } else {
        if (tab.r_global) {
            st.work.rbuf.reserve(8 * (size_t)std::max<int64_t>(centers, 1) * tab.rsize, "coefficient scratch");
            p.rbuf = st.work.rbuf.as<double>();
        }
        if (centers > 0 && tab.edge_cap > 0 && !variant->paired) {
            // Centre kernel on edge lists: per chunk, the walk-only kernel
            // fills the slots, then the centre kernel reads them.
            const int64_t chunk = std::min<int64_t>(centers, edge_chunk);
            const size_t slots = (size_t)std::max<int64_t>(chunk, 1);
            st.work.edges.reserve(slots * (size_t)tab.edge_cap * sizeof(double4), "edge slots");
            st.work.edge_info.reserve(slots * (size_t)tab.edge_cap * sizeof(int32_t), "edge slots");
            st.work.edge_count.reserve(slots * sizeof(int32_t), "edge counts");
            p.edges = st.work.edges.as<double4>();
            p.edge_info = st.work.edge_info.as<int32_t>();
            p.edge_count = st.work.edge_count.as<int32_t>();
            SoapTables walk_tab = tab;
            walk_tab.warp_bytes = paired::kHeaderBytes;
            for (int64_t c0 = a0; c0 < a1; c0 += chunk) {
                p.grid_begin = c0;
                p.grid_end = std::min(a1, c0 + chunk);
                const int64_t one_per_warp = (p.grid_end - c0 + kWarps - 1) / kWarps;
                NvtxRange range("mdsoap walk + expansion");
                walk_launch(dim3((unsigned)std::min(one_per_warp, std::max<int64_t>(st.walk_grid, 1))), walk_smem,
                            stream, walk_tab, p);
                check(cudaGetLastError(), "walk kernel launch");
                variant->center(dim3((unsigned)one_per_warp), center_smem, stream, tab, p);
                check(cudaGetLastError(), "centre kernel launch");
                launches.fetch_add(2, std::memory_order_relaxed);
            }
            p.grid_begin = a0;
            p.grid_end = a1;
            p.edges = nullptr;
            p.edge_info = nullptr;
            p.edge_count = nullptr;
        } else if (centers > 0) {
            int64_t grid = (centers + kWarps - 1) / kWarps;
            if (variant->paired && st.center_grid > 0) grid = std::min(grid, st.center_grid);
            NvtxRange range("mdsoap expansion");
            variant->center(dim3((unsigned)grid), center_smem, stream, tab, p);
            check(cudaGetLastError(), "centre kernel launch");
            launches.fetch_add(1, std::memory_order_relaxed);
        }
    }
    if (after_center) check(cudaEventRecord(after_center, stream), "timing event");
    if (average != MDSOAP_AVERAGE_OFF && s1 > s0) {
        variant->structure(dim3((unsigned)(s1 - s0)), structure_smem, stream, tab, b.offsets, s0, s1, p.cbuf, p.pbuf,
                           out, s0);
        check(cudaGetLastError(), "structure kernel launch");
        launches.fetch_add(1, std::memory_order_relaxed);
    }
}

namespace {

void validate_host_batch(const mdsoap_plan* plan, const mdsoap_batch& b) {
    // detail/batch.hpp:19-80 (validate_batch) and species.hpp:55-69 (validate_species).
    if (b.structures < 0 || b.atoms < 0 || b.offsets == nullptr) raise(MDSOAP_INVALID_ARGUMENT, "invalid structure batch");
    if (b.structures == 0) {
        if (b.atoms != 0 || b.offsets[0] != 0)
            raise(MDSOAP_INVALID_ARGUMENT, "empty structure batch has non-empty atom data");
        return;
    }
    if (!b.numbers || !b.positions || !b.cells || !b.pbc)
        raise(MDSOAP_INVALID_ARGUMENT, "structure batch contains null arrays");
    if (b.offsets[0] != 0 || b.offsets[b.structures] != b.atoms)
        raise(MDSOAP_INVALID_ARGUMENT, "offsets do not describe the flattened arrays");
    if (b.atoms > 2147483647LL) raise(MDSOAP_INVALID_ARGUMENT, "neighbor atom index exceeds int32 range");
    for (int64_t s = 0; s < b.structures; ++s) {
        if (b.offsets[s] < 0 || b.offsets[s] > b.offsets[s + 1] || b.offsets[s + 1] > b.atoms)
            raise(MDSOAP_INVALID_ARGUMENT, "offsets must be monotonic");
        bool periodic = true, isolated = true;
        for (int a = 0; a < 3; ++a) {
            const int32_t f = b.pbc[3 * s + a];
            if (f != 0 && f != 1) raise(MDSOAP_INVALID_ARGUMENT, "pbc must contain only 0 or 1");
            periodic = periodic && f == 1;
            isolated = isolated && f == 0;
        }
        if (!periodic && !isolated)
            raise(MDSOAP_INVALID_ARGUMENT, "mixed periodicity is not supported; use all-zero or all-one pbc");
        const double* c = b.cells + 9 * s;
        for (int k = 0; k < 9; ++k)
            if (!std::isfinite(c[k])) raise(MDSOAP_INVALID_ARGUMENT, "cells must be finite");
        const double det = c[0] * (c[4] * c[8] - c[5] * c[7]) - c[1] * (c[3] * c[8] - c[5] * c[6]) +
                           c[2] * (c[3] * c[7] - c[4] * c[6]);
        if (periodic && (!std::isfinite(det) || std::abs(det) < 1e-14))
            raise(MDSOAP_INVALID_ARGUMENT, "cells must be nonsingular");
    }
    for (int64_t a = 0; a < b.atoms; ++a) {
        if (b.numbers[a] <= 0) raise(MDSOAP_INVALID_ARGUMENT, "atomic numbers must be positive");
        for (int c = 0; c < 3; ++c)
            if (!std::isfinite(b.positions[3 * a + c])) raise(MDSOAP_INVALID_ARGUMENT, "positions must be finite");
        if (!plan) continue;
        bool known = false;
        for (int32_t z : plan->species) known = known || z == b.numbers[a];
        if (!known) raise(MDSOAP_INVALID_ARGUMENT, "batch contains an atomic number outside calculator species");
    }
}

// Host copy with several threads (pinned staging -> caller memory).
void parallel_copy(char* dst, const char* src, size_t bytes) {
    const size_t grain = (size_t)32 << 20;
    const unsigned hw = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
    const size_t parts = std::min<size_t>(hw, (bytes + grain - 1) / grain);
    if (parts <= 1) {
        std::memcpy(dst, src, bytes);
        return;
    }
    std::vector<std::thread> threads;
    const size_t step = (bytes + parts - 1) / parts;
    for (size_t i = 0; i < parts; ++i) {
        const size_t begin = i * step;
        const size_t end = std::min(bytes, begin + step);
        if (begin >= end) break;
        threads.emplace_back([=] { std::memcpy(dst + begin, src + begin, end - begin); });
    }
    for (auto& t : threads) t.join();
}

bool is_pinned(const void* ptr) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeHost;
}

int64_t block_bytes_target() {
    const char* env = std::getenv("MDSOAP_BLOCK_BYTES");
    if (env) {
        const long long v = std::atoll(env);
        if (v > 0) return v;
    }
    return (int64_t)64 << 20;
}

}  // namespace

// One device's share [s0, s1) of a host batch, copied into `out` (rows of the shard).
void mdsoap_plan::shard_compute(int device, const mdsoap_batch& batch, int64_t s0, int64_t s1, char* out,
                                mdsoap_cancel_fn cancel, void* ctx, std::atomic<bool>& stop) {
    DeviceState& st = state(device);
    std::lock_guard<std::mutex> lock(st.mutex);
    check(cudaSetDevice(device), "cudaSetDevice");
    const int64_t a_begin = batch.offsets[s0];
    const int64_t structures = s1 - s0;
    const int64_t atoms = batch.offsets[s1] - a_begin;
    const bool by_structure = average != MDSOAP_AVERAGE_OFF;
    const size_t row_bytes = (size_t)features * out_elem();
    // Upload the shard (offsets rebased to the shard).
    Workspace& w = st.work;
    w.numbers.reserve(4 * (size_t)std::max<int64_t>(atoms, 1), "numbers");
    w.positions.reserve(24 * (size_t)std::max<int64_t>(atoms, 1), "positions");
    w.cells.reserve(72 * (size_t)std::max<int64_t>(structures, 1), "cells");
    w.pbc.reserve(12 * (size_t)std::max<int64_t>(structures, 1), "pbc");
    w.offsets.reserve(8 * (size_t)(structures + 1), "offsets");
    std::vector<int64_t> offsets(structures + 1);
    for (int64_t s = 0; s <= structures; ++s) offsets[s] = batch.offsets[s0 + s] - a_begin;
    cudaStream_t cs = st.compute;
    NvtxRange upload_range("mdsoap upload");
    if (atoms > 0) {
        check(cudaMemcpyAsync(w.numbers.ptr, batch.numbers + a_begin, 4 * atoms, cudaMemcpyHostToDevice, cs), "H2D numbers");
        check(cudaMemcpyAsync(w.positions.ptr, batch.positions + 3 * a_begin, 24 * atoms, cudaMemcpyHostToDevice, cs),
              "H2D positions");
    }
    check(cudaMemcpyAsync(w.cells.ptr, batch.cells + 9 * s0, 72 * structures, cudaMemcpyHostToDevice, cs), "H2D cells");
    check(cudaMemcpyAsync(w.pbc.ptr, batch.pbc + 3 * s0, 12 * structures, cudaMemcpyHostToDevice, cs), "H2D pbc");
    check(cudaMemcpyAsync(w.offsets.ptr, offsets.data(), 8 * (structures + 1), cudaMemcpyHostToDevice, cs),
          "H2D offsets");
    DeviceBatch db{w.numbers.as<int32_t>(), w.positions.as<double>(), w.cells.as<double>(), w.pbc.as<int32_t>(),
                   w.offsets.as<int64_t>(), structures, atoms};
    unsigned* error = st.error.as<unsigned>();
    check(cudaMemsetAsync(error, 0, sizeof(unsigned), cs), "clear error word");
    bin(st, db, cs, error);

    // Blocks of whole structures, about block_bytes_target() of output each.
    const int64_t target = std::max<int64_t>(1, block_bytes_target() / (int64_t)std::max<size_t>(row_bytes, 1));
    std::vector<int64_t> cuts{0};
    {
        int64_t rows = 0;
        for (int64_t s = 0; s < structures; ++s) {
            rows += by_structure ? 1 : offsets[s + 1] - offsets[s];
            if (rows >= target) {
                cuts.push_back(s + 1);
                rows = 0;
            }
        }
        if (cuts.back() != structures) cuts.push_back(structures);
    }
    const bool direct = is_pinned(out);
    size_t max_block_bytes = 0;
    for (size_t i = 0; i + 1 < cuts.size(); ++i) {
        const int64_t rows = by_structure ? cuts[i + 1] - cuts[i] : offsets[cuts[i + 1]] - offsets[cuts[i]];
        max_block_bytes = std::max(max_block_bytes, (size_t)rows * row_bytes);
    }
    for (int i = 0; i < 2; ++i) {
        st.out[i].reserve(std::max<size_t>(max_block_bytes, 16), "output block");
        if (!direct) st.staging[i].reserve(std::max<size_t>(max_block_bytes, 16));
    }
    const size_t blocks = cuts.size() - 1;
    struct Pending {
        size_t bytes;
        char* dst;
    };
    std::vector<Pending> pending(blocks);
    auto finish = [&](size_t i) {
        check(cudaEventSynchronize(st.copied[i % 2]), "D2H wait");
        if (!direct && pending[i].bytes) parallel_copy(pending[i].dst, static_cast<char*>(st.staging[i % 2].ptr), pending[i].bytes);
    };
    for (size_t i = 0; i < blocks; ++i) {
        if (stop.load() || (cancel && cancel(ctx))) {
            stop.store(true);
            if (i > 0) finish(i - 1);
            check(cudaStreamSynchronize(cs), "cancel sync");
            raise(MDSOAP_CANCELLED, "descriptor computation was cancelled");
        }
        const int64_t bs0 = cuts[i], bs1 = cuts[i + 1];
        const int64_t rows = by_structure ? bs1 - bs0 : offsets[bs1] - offsets[bs0];
        const int64_t row0 = by_structure ? bs0 : offsets[bs0];
        const size_t bytes = (size_t)rows * row_bytes;
        char* dst = out + (size_t)row0 * row_bytes;
        if (i >= 2) check(cudaStreamWaitEvent(cs, st.copied[i % 2], 0), "wait output buffer");
        run_block(st, db, bs0, bs1, offsets[bs0], offsets[bs1], st.out[i % 2].ptr, cs, error);
        check(cudaEventRecord(st.computed[i % 2], cs), "record compute");
        if (i >= 1) finish(i - 1);
        check(cudaStreamWaitEvent(st.copy, st.computed[i % 2], 0), "wait compute");
        if (bytes) {
            NvtxRange range("mdsoap D2H");
            check(cudaMemcpyAsync(direct ? dst : st.staging[i % 2].ptr, st.out[i % 2].ptr, bytes, cudaMemcpyDeviceToHost,
                                  st.copy),
                  "D2H output");
        }
        check(cudaEventRecord(st.copied[i % 2], st.copy), "record copy");
        pending[i] = {bytes, dst};
    }
    if (blocks) finish(blocks - 1);
    check(cudaStreamSynchronize(cs), "compute sync");
    unsigned bits = 0;
    check(cudaMemcpy(&bits, error, sizeof(unsigned), cudaMemcpyDeviceToHost), "read error word");
    if (bits) raise(bits & kErrUnknownSpecies || bits & kErrMixedPbc || bits & kErrSingularCell ? MDSOAP_INVALID_ARGUMENT
                                                                                                : MDSOAP_INTERNAL,
                    device_error_text(bits));
}

struct mdsoap_graph {
    int64_t atoms = 0;
    std::vector<int64_t> offsets;
    std::vector<int32_t> atom_ids, shifts;
    std::vector<double> displacements, distance2;
};

struct mdsoap_pairs {
    std::vector<double> records;      // [pairs][5]
    std::vector<double> values;       // [pairs][4]
    std::vector<int64_t> row_offsets; // [structures + 1]
};

// ---------------------------------------------------------------------------
// C ABI

extern "C" {

const char* mdsoap_last_error(void) { return g_error.c_str(); }

int32_t mdsoap_abi_version(void) { return MDSOAP_ABI_VERSION; }

int32_t mdsoap_device_count(void) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return count;
}

int mdsoap_plan_create(const mdsoap_params* params, mdsoap_plan** plan_out) {
    if (!params || !plan_out) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    *plan_out = nullptr;
    const mdsoap_params& q = *params;
    // soap.cpp:1149-1176 parameter checks; n_max <= 32 is the reference CUDA
    // plugin's limit (extended_descriptors_soap.cuh:812-815).
    if (q.n_species < 1 || q.n_species > kMaxSpecies || !q.species)
        return fail(MDSOAP_INVALID_ARGUMENT, "SOAP species must contain 1..64 atomic numbers");
    if (!std::isfinite(q.r_cut) || !std::isfinite(q.sigma) || q.r_cut <= 0.0 || q.sigma <= 0.0 || q.n_max < 1 ||
        q.l_max < 0 || q.l_max > kMaxL)
        return fail(MDSOAP_INVALID_ARGUMENT, "invalid SOAP parameters");
    if (q.n_max > kMaxN) return fail(MDSOAP_INVALID_ARGUMENT, "invalid CUDA SOAP parameters (n_max > 32)");
    if (q.average < 0 || q.average > 2) return fail(MDSOAP_INVALID_ARGUMENT, "unsupported CUDA SOAP average mode");
    if (q.output_dtype != MDSOAP_FLOAT32 && q.output_dtype != MDSOAP_FLOAT64)
        return fail(MDSOAP_INVALID_ARGUMENT, "output dtype must be float32 or float64");
    if (q.compression < MDSOAP_COMPRESSION_OFF || q.compression > MDSOAP_COMPRESSION_CROSSOVER)
        return fail(MDSOAP_INVALID_ARGUMENT, "unsupported CUDA SOAP compression");
    // soap.cpp:1198-1210 weighting checks.
    if (q.weighting_function < MDSOAP_WEIGHTING_NONE || q.weighting_function > MDSOAP_WEIGHTING_EXP)
        return fail(MDSOAP_INVALID_ARGUMENT, "unsupported CUDA SOAP weighting");
    if (q.weighting_function != MDSOAP_WEIGHTING_NONE &&
        (!std::isfinite(q.weighting_r0) || q.weighting_r0 <= 0.0 || !std::isfinite(q.weighting_c) ||
         q.weighting_c < 0.0 || !std::isfinite(q.weighting_d) || q.weighting_d < 0.0 ||
         !std::isfinite(q.weighting_m) || q.weighting_m < 0.0))
        return fail(MDSOAP_INVALID_ARGUMENT, "invalid SOAP weighting parameters");
    if (q.weighting_has_w0 && (!std::isfinite(q.weighting_w0) || q.weighting_w0 < 0.0))
        return fail(MDSOAP_INVALID_ARGUMENT, "invalid SOAP w0 weighting");
    if (q.radial_basis != MDSOAP_RADIAL_GTO && q.radial_basis != MDSOAP_RADIAL_POLYNOMIAL)
        return fail(MDSOAP_INVALID_ARGUMENT, "unsupported CUDA SOAP radial basis");
    const bool polynomial = q.radial_basis == MDSOAP_RADIAL_POLYNOMIAL;
    if (!polynomial && (!q.alphas || !q.betas)) return fail(MDSOAP_INVALID_ARGUMENT, "invalid SOAP radial basis size");
    // soap.cpp:1165-1192 polynomial basis checks; 128 nodes is this library's limit.
    if (polynomial && (q.radial_grid_size < 2 || q.radial_grid_size > kMaxGrid || !q.radial_grid ||
                       !q.radial_weights || !q.radial_values))
        return fail(MDSOAP_INVALID_ARGUMENT, "invalid SOAP polynomial radial basis size");
    if (polynomial) {
        const int Q = q.radial_grid_size;
        for (int i = 0; i < Q; ++i)
            if (!std::isfinite(q.radial_grid[i]) || q.radial_grid[i] < 0.0 || q.radial_grid[i] > q.r_cut)
                return fail(MDSOAP_INVALID_ARGUMENT, "SOAP polynomial radial grid must be finite and in range");
        for (int i = 0; i < Q; ++i)
            if (!std::isfinite(q.radial_weights[i]) || q.radial_weights[i] <= 0.0)
                return fail(MDSOAP_INVALID_ARGUMENT, "SOAP polynomial radial weights must be positive and finite");
        for (int i = 0; i < Q * q.n_max; ++i)
            if (!std::isfinite(q.radial_values[i]))
                return fail(MDSOAP_INVALID_ARGUMENT, "SOAP polynomial radial basis must be finite");
    }
    for (int i = 0; i < q.n_species; ++i) {
        if (q.species[i] <= 0) return fail(MDSOAP_INVALID_ARGUMENT, "species must be positive atomic numbers");
        for (int j = 0; j < i; ++j)
            if (q.species[j] == q.species[i]) return fail(MDSOAP_INVALID_ARGUMENT, "species must be unique");
    }
    try {
        auto plan = std::make_unique<mdsoap_plan>();
        plan->n_species = q.n_species;
        plan->n_max = q.n_max;
        plan->l_max = q.l_max;
        plan->average = q.average;
        plan->out_dtype = q.output_dtype;
        plan->r_cut = q.r_cut;
        plan->sigma = q.sigma;
        plan->species.assign(q.species, q.species + q.n_species);
        plan->weights.assign(q.n_species, 1.0);
        if (q.species_weights) {
            for (int i = 0; i < q.n_species; ++i) {
                if (!std::isfinite(q.species_weights[i]))
                    return fail(MDSOAP_INVALID_ARGUMENT, "SOAP species weights must be finite");
                plan->weights[i] = q.species_weights[i];
            }
        }
        const int L = q.l_max, n = q.n_max, W = L + 1;
        if (polynomial) {
            // The projection needs no beta transform and no pi^{3/2}: the plan
            // carries identity betas and unit radial items for the shared tail.
            plan->alphas.assign(W * n, 0.0);
            plan->betas.assign(W * n * n, 0.0);
            for (int l = 0; l < W; ++l)
                for (int k = 0; k < n; ++k) plan->betas[(l * n + k) * n + k] = 1.0;
            // prepare_soap (soap.cpp:555-569): wv[q][n] = weight_q grid_q^2 values[n][q].
            const int Q = q.radial_grid_size;
            plan->poly.assign(q.radial_grid, q.radial_grid + Q);
            plan->poly.resize((size_t)Q * (n + 1));
            for (int i = 0; i < Q; ++i) {
                const double quad = q.radial_weights[i] * q.radial_grid[i] * q.radial_grid[i];
                for (int k = 0; k < n; ++k) plan->poly[Q + (size_t)i * n + k] = quad * q.radial_values[(size_t)k * Q + i];
            }
        } else {
            plan->alphas.assign(q.alphas, q.alphas + W * n);
            plan->betas.assign(q.betas, q.betas + W * n * n);
        }
        for (double v : plan->alphas)
            if (!std::isfinite(v)) return fail(MDSOAP_INVALID_ARGUMENT, "SOAP radial basis must be finite");
        for (double v : plan->betas)
            if (!std::isfinite(v)) return fail(MDSOAP_INVALID_ARGUMENT, "SOAP radial basis must be finite");
        // soap.cpp:1214 + neighbor.cpp:552 (host double arithmetic, same order).
        const double padding = q.sigma * std::sqrt(-2.0 * std::log(1e-3));
        plan->cutoff = q.r_cut + padding;
        // prepare_soap (soap.cpp:507-534).
        const double eta = 1.0 / (2.0 * q.sigma * q.sigma);
        std::vector<double> eta_powers(W, 1.0);
        for (int l = 1; l <= L; ++l) eta_powers[l] = eta_powers[l - 1] * eta;
        for (int l = L; l >= 0; --l) {
            for (int k = 0; k < n; ++k) {
                const double alpha = plan->alphas[l * n + k];
                const double denominator = alpha + eta;
                RadialItem it;
                it.prefactor = eta_powers[l] * std::pow(denominator, -l - 1.5);
                it.exponent = alpha * eta / denominator;
                it.l = l;
                it.k = k;
                plan->items.push_back(it);
            }
        }
        SoapTables& t = plan->tab;
        std::memset(&t, 0, sizeof(t));
        t.n_species = q.n_species;
        t.n_max = n;
        t.l_max = L;
        t.H = W * W;
        t.items = W * n;
        // mu2 pools every species into one density (soap.cpp:613-615).
        const int coef_species = q.compression == MDSOAP_COMPRESSION_MU2 ? 1 : q.n_species;
        t.rows = coef_species * n;
        t.coef_species = coef_species;
        t.compression = q.compression;
        plan->compression = q.compression;
        const int64_t width = (int64_t)q.n_species * n;
        switch (q.compression) {  // soap_features, soap.cpp:373-387
            case MDSOAP_COMPRESSION_MU2: plan->features = (int64_t)n * (n + 1) / 2 * W; break;
            case MDSOAP_COMPRESSION_MU1NU1: plan->features = (int64_t)q.n_species * n * n * W; break;
            case MDSOAP_COMPRESSION_CROSSOVER: plan->features = (int64_t)q.n_species * n * (n + 1) / 2 * W; break;
            default: plan->features = width * (width + 1) / 2 * W;
        }
        t.features = plan->features;
        t.weight_fn = q.weighting_function;
        t.has_w0 = q.weighting_has_w0 ? 1 : 0;
        t.w_r0 = q.weighting_r0;
        t.w_c = q.weighting_c;
        t.w_d = q.weighting_d;
        t.w_m = q.weighting_m;
        t.w_0 = q.weighting_w0;
        // Per-edge weights: a weighting function or w0, and mu2 (the species
        // weight then multiplies each edge of the pooled density).
        t.weighted = (t.weight_fn != 0 || t.has_w0 || q.compression == MDSOAP_COMPRESSION_MU2) ? 1 : 0;
        t.average = q.average;
        t.out_f64 = q.output_dtype == MDSOAP_FLOAT64;
        t.cutoff2 = plan->cutoff * plan->cutoff;
        const double pi = 3.141592653589793238462643383279502884;
        t.soap_scale = polynomial ? 1.0 : pi * std::sqrt(pi);
        t.grid_size = polynomial ? q.radial_grid_size : 0;
        t.eta = eta;
        for (int l = 0; l <= L; ++l) {
            t.power_pref[l] = pi * std::sqrt(8.0 / (2.0 * l + 1.0));
            for (int m = 0; m <= l; ++m) {
                const int i = l * (l + 1) / 2 + m;
                // solid_harmonic_normalization (soap.cpp:26-38), sqrt 2 folded in for m > 0.
                const double norm =
                    std::sqrt((2.0 * l + 1.0) / (4.0 * pi) * std::exp(std::lgamma(l - m + 1.0) - std::lgamma(l + m + 1.0)));
                t.ynorm[i] = m == 0 ? norm : norm * 1.414213562373095048801688724209698079;
                t.yra[i] = l > m ? (2.0 * l - 1.0) / (l - m) : 0.0;
                t.yrb[i] = l > m ? (l + m - 1.0) / (l - m) : 0.0;
            }
        }
        for (int i = 0; i < q.n_species; ++i) t.species_weight[i] = plan->weights[i];
        // Kernel choice.  The paired-channel kernel is the default where it
        // applies: its scaled_exp needs every radial factor P exp(-E r^2),
        // r <= cutoff, to be a normal double with E r^2 <= 708.  MDSOAP_VARIANT=k
        // (tuning knob) picks the k-th of [paired kernel if it applies, the
        // class's kernels...] instead; an index past the list gives the default.
        bool radial_normal = true;
        for (const RadialItem& it : plan->items) {
            const double span = it.exponent * t.cutoff2;
            if (!(it.prefactor > 0.0) || !std::isfinite(it.prefactor) || !(it.exponent >= 0.0) || !(span <= 700.0) ||
                std::log(it.prefactor) - span < -690.0)
                radial_normal = false;
        }
        const Variant* paired = polynomial ? poly_variant(n, L)
                                : radial_normal ? paired_variant(n, L, q.output_dtype == MDSOAP_FLOAT64,
                                                                 (q.compression == MDSOAP_COMPRESSION_MU2 ? 1
                                                                                                          : q.n_species) *
                                                                     (q.output_dtype == MDSOAP_FLOAT64 ? 2 : 1))
                                                : nullptr;
        const char* env = std::getenv("MDSOAP_VARIANT");
        const int want = env ? std::atoi(env) : -1;
        const Variant* picked = nullptr;
        if (paired && want <= 0) picked = paired;
        else picked = &pick_variant(n, L, paired ? want - 1 : want);
        const bool needs_paired = t.weighted || q.compression != MDSOAP_COMPRESSION_OFF || polynomial;
        if (needs_paired && paired) picked = paired;
        if (paired && picked != paired && want > 0 && want - 1 >= 0) {
            // An index past the class list falls back to the default (the paired kernel).
            int members = 0;
            for (const Variant& cv : kVariants) members += cv.cls == variant_class(n, L);
            if (want - 1 >= members) picked = paired;
        }
        if (picked->paired) {
            const Variant& v = *picked;
            plan->variant = &v;
            // The full-accuracy (float64-row) instantiations keep every
            // species' neighbour sum as two partial sums: half-length sums,
            // the accuracy class of the reference's two-lane SIMD reduction.
            t.ksplit = v.precise ? 2 : 1;
            t.type_groups = (coef_species + v.maxt / t.ksplit - 1) / (v.maxt / t.ksplit);
            t.slot_groups = 1;
            t.beta_in_smem = 1;
            t.csize = coef_species * n * W * (W + 1);
            t.hp = W * (W + 1);
            t.rs = mma::row_stride(L);
            t.rsize = coef_species * n * t.rs;
            t.n_magic = n == 1 ? 0u : (uint32_t)((1ull << 32) / (uint64_t)n + 1ull);
            const bool single_pass = t.type_groups == 1;
            const size_t grid_bytes = polynomial ? ((size_t)t.grid_size * 9 * 8 + 15) & ~(size_t)15 : 0;
            const size_t flir_bytes = polynomial ? (size_t)W * t.grid_size * 8 : 0;
            const size_t shared = 256 + (size_t)W * 64 * 8 + grid_bytes;
            // paired::Layout<L>::ROW: G views of 2L+2 doubles, padded to = 2 (mod 4).
            const size_t views = (size_t)(1 + (L + 1) / 2) * (size_t)(2 * L + 2);
            const size_t row = views + (2 - views % 4 + 4) % 4;
            const size_t r_bytes = (size_t)t.rsize * 8;
            auto align16 = [](size_t x) { return (x + 15) & ~(size_t)15; };
            auto walk = [&](int c) { return (size_t)paired::kHeaderBytes + (size_t)c * row * 8 + flir_bytes; };
            auto per_warp = [&](int c, bool r_in) {
                if (!r_in) return align16(walk(c));
                if (single_pass) return align16(std::max(walk(c), r_bytes));
                return align16(walk(c)) + align16(r_bytes);
            };
            const size_t budget = 228 * 1024 / (size_t)v.minb - 1024, budget1 = 227 * 1024;
            int chunk = 32;
            bool r_smem = true;
            while (chunk > 8 && shared + kWarps * per_warp(chunk, true) > budget) chunk -= 8;
            if (shared + kWarps * per_warp(chunk, true) > budget1) {
                r_smem = false;
                chunk = 32;
                while (chunk > 8 && shared + kWarps * per_warp(chunk, false) > budget) chunk -= 8;
            }
            t.chunk = chunk;
            t.r_global = r_smem ? 0 : 1;
            t.warp_bytes = (int32_t)per_warp(chunk, r_smem);
            t.r_offset = (r_smem && !single_pass) ? (int32_t)align16(walk(chunk)) : 0;
            plan->center_smem = shared + kWarps * (size_t)t.warp_bytes;
            plan->structure_smem = q.average == MDSOAP_AVERAGE_INNER ? (size_t)t.csize * 8 : 0;
            plan->csize = t.csize;
            // n_max == 8 tails in registers run as their own kernel (soap_tail_kernel).
            // MDSOAP_SPLIT_TAIL=0 keeps them fused (measurement knob).
            const char* split_env = std::getenv("MDSOAP_SPLIT_TAIL");
            const bool split_allowed = !(split_env && split_env[0] == '0');
            const size_t generic_smem = (size_t)W * 64 * 8 + (size_t)kWarps * t.rsize * 8;  // beta + a block per warp
            const bool regs = n == 8 && coef_species * t.ksplit <= v.maxt;
            if (split_allowed && !polynomial && q.average != MDSOAP_AVERAGE_INNER && r_smem &&
                (regs || generic_smem <= budget1)) {
                // Register tail (soap_tail_kernel) where the coefficients fit
                // the register banks, else soap_tail_generic_kernel.
                t.split_tail = regs ? 1 : 2;
                plan->tail_smem = regs ? (size_t)W * 64 * 8 + 2 * (size_t)t.rsize * 8  // beta + two coefficient blocks
                                       : generic_smem;
                // The raw-sum scratch holds one block per centre of a chunk:
                // chunks of at most 4 GiB (240 k centres for config 2's
                // 17 KB blocks, so config 2 runs as one pair of launches).
                plan->tail_chunk = std::max<int64_t>(4096, (int64_t)((4ull << 30) / (8ull * (uint64_t)t.rsize)));
                // Edge-list split: a walk-only kernel writes each centre's
                // accepted edges (36 B each) to a slot of edge_cap edges, an
                // expansion-only kernel reads them, and the fused kernel
                // redoes the centres whose slot overflowed.  Slots of a
                // chunk take at most 4 GiB too.  MDSOAP_EDGE_CAP sets the
                // slot size (0: walk and expansion in one kernel).
                int64_t cap = 512;
                if (const char* cap_env = std::getenv("MDSOAP_EDGE_CAP")) cap = std::max<int64_t>(0, std::atoll(cap_env));
                // (Float32 rows: the expansion kernel pairs radial indices k and
                // k + n_max / 2, so n_max must be even.)
                if (cap > 0 && v.walk && v.expand && (v.precise || n % 2 == 0)) {
                    t.edge_cap = (int32_t)std::min<int64_t>(cap, 1 << 20);
                    t.parity_group = std::max(1, v.maxt / t.ksplit);
                    plan->walk_launch = v.walk;
                    plan->walk_symbol = v.walk_sym;
                    plan->walk_smem = 256 + 64 * 8 + (size_t)kWarps * paired::kHeaderBytes;
                    // The expansion-only kernel: one species per pass (two
                    // banks of partial sums for float64 rows), so few
                    // registers (168: 3 CTAs per SM, against 2 for the fused
                    // kernel); the raw sums go straight to the tail's
                    // scratch; the largest edge chunk whose shared memory
                    // fits 3 CTAs per SM.
                    plan->expand_launch = v.expand;
                    plan->expand_symbol = v.expand_sym;
                    const size_t ebudget = 228 * 1024 / 3 - 1024;
                    int echunk = 32;
                    auto ewarp = [&](int c) { return align16((size_t)paired::kHeaderBytesExpand + (size_t)c * row * 8); };
                    // exp table only: no beta table in this kernel
                    const size_t eshared = (size_t)paired::exp_table_bytes(2, v.precise);
                    while (echunk > 8 && eshared + kWarps * ewarp(echunk) > ebudget) echunk -= 8;
                    plan->expand_chunk = echunk;
                    plan->expand_warp_bytes = (int32_t)ewarp(echunk);
                    plan->expand_smem = eshared + kWarps * ewarp(echunk);
                    const int64_t slot_bytes = (int64_t)t.edge_cap * (int64_t)(sizeof(double4) + sizeof(int32_t)) + 4;
                    plan->tail_chunk = std::min<int64_t>(plan->tail_chunk,
                                                         std::max<int64_t>(4096, (int64_t)(4ull << 30) / slot_bytes));
                }
                if (const char* chunk_env = std::getenv("MDSOAP_TAIL_CHUNK"))
                    plan->tail_chunk = std::max<int64_t>(kWarps, std::atoll(chunk_env));
            }
            plan->kernel_label = v.name;
            if (t.edge_cap > 0) {
                const std::string prec = v.precise ? "true" : "false";
                plan->kernel_label = "soap_paired_kernel<1, 0, " + prec + ", 4, walk> + soap_paired_kernel<" +
                                     (v.precise ? "2" : "1") + ", " + std::to_string(L) + ", " + prec +
                                     ", 3, expand> (edge lists; overflowed slots: " + v.name + ")";
            }
            if (t.split_tail == 1)
                plan->kernel_label += " + soap_tail_kernel<" + std::to_string(L) + ", " + std::to_string(v.maxt) + ">";
            else if (t.split_tail == 2)
                plan->kernel_label += " + soap_tail_generic_kernel<" + std::to_string(L) + ">";
            if (plan->center_smem > budget1 || plan->structure_smem > budget1)
                return fail(MDSOAP_INVALID_ARGUMENT, "SOAP parameters need more shared memory than the device offers");
            *plan_out = plan.release();
            return MDSOAP_OK;
        }
        if (polynomial)
            return fail(MDSOAP_INVALID_ARGUMENT,
                        "the SOAP polynomial radial basis runs on the paired-channel kernel, which needs "
                        "n_max <= 8, n_max (1 + (l_max + 1) / 2) <= 32 and l_max <= 6");
        const Variant& sv = *picked;
        plan->variant = &sv;
        const int ns = (sv.l0 > 0) + (sv.l1 > 0) + (sv.l2 > 0);
        const int slots = (t.items + 31) / 32;
        t.slot_groups = (slots + ns - 1) / ns;
        t.ksplit = 1;
        t.type_groups = (coef_species + sv.maxt - 1) / sv.maxt;
        const bool single_pass = t.slot_groups == 1 && t.type_groups == 1;
        // One-warp scalar kernels with n_max <= 8 finish on the tensor cores:
        // row-strided coefficient block, padded 8 x 8 beta table in shared memory.
        const bool mma_tail = sv.nmax <= 8;
        const size_t beta_bytes = mma_tail ? (size_t)W * 64 * 8 : (size_t)W * n * n * 8;
        t.beta_in_smem = mma_tail || beta_bytes <= 32768;
        // CTA-shared: 32-entry exp table (256 B) + optional beta copy.
        const size_t beta_smem = 256 + (t.beta_in_smem ? ((beta_bytes + 15) & ~(size_t)15) : 0);
        t.csize = coef_species * n * W * (W + 1);
        t.hp = W * (W + 1);
        t.rs = mma_tail ? mma::row_stride(L) : 0;
        t.rsize = mma_tail ? coef_species * n * t.rs : t.csize;
        t.n_magic = n == 1 ? 0u : (uint32_t)((1ull << 32) / (uint64_t)n + 1ull);
        const size_t r_bytes = (size_t)t.rsize * 8;
        // Pending edges: dx dy dz r2 weight (doubles) + species (int32).
        const size_t pend = kRegionHeader + (size_t)kPending * 44;
        auto region_a = [&](int chunk) { return pend + ((size_t)chunk * t.hp + 48) * 8; };
        auto align16 = [](size_t x) { return (x + 15) & ~(size_t)15; };
        auto per_warp = [&](int chunk, bool r_in_smem) {
            if (!r_in_smem) return align16(region_a(chunk));
            if (single_pass) return align16(std::max(region_a(chunk), r_bytes));
            return align16(region_a(chunk)) + align16(r_bytes);
        };
        // Largest chunk (<= 32) that lets the variant's MINB CTAs share an SM
        // (228 KB per SM, 1 KB reserved per CTA); failing that, the smallest
        // footprint that fits one CTA, with the coefficient blocks moved to
        // global scratch if they alone are too large.
        const size_t budget = 228 * 1024 / (size_t)sv.minb - 1024, budget1 = 227 * 1024;
        int chunk = 32;
        bool r_smem = true;
        while (chunk > 8 && beta_smem + kWarps * per_warp(chunk, true) > budget) chunk -= 8;
        if (beta_smem + kWarps * per_warp(chunk, true) > budget1) {
            r_smem = false;
            chunk = 32;
            while (chunk > 8 && beta_smem + kWarps * per_warp(chunk, false) > budget) chunk -= 8;
        }
        t.chunk = chunk;
        t.r_global = r_smem ? 0 : 1;
        t.warp_bytes = (int32_t)per_warp(chunk, r_smem);
        t.r_offset = (r_smem && !single_pass) ? (int32_t)align16(region_a(chunk)) : 0;
        plan->center_smem = beta_smem + kWarps * (size_t)t.warp_bytes;
        plan->structure_smem = q.average == MDSOAP_AVERAGE_INNER ? (size_t)t.csize * 8 : 0;
        plan->csize = t.csize;
        {
            // Edge lists: the paired walk-only kernel (prefiltered candidates,
            // float32 rows with certified pairs) writes each centre's accepted
            // edges to a slot that the centre kernel reads instead of walking
            // (centres whose slot overflowed walk themselves).  Slots of a
            // chunk take at most 4 GiB.  MDSOAP_EDGE_CAP as for the paired plans.
            int64_t cap = 512;
            if (const char* cap_env = std::getenv("MDSOAP_EDGE_CAP")) cap = std::max<int64_t>(0, std::atoll(cap_env));
            if (cap > 0) {
                const bool f64 = q.output_dtype == MDSOAP_FLOAT64;
                t.edge_cap = (int32_t)std::min<int64_t>(cap, 1 << 20);
                plan->walk_launch = f64 ? &launch::paired_walk<true> : &launch::paired_walk<false>;
                plan->walk_symbol = f64 ? &launch::paired_walk_symbol<true> : &launch::paired_walk_symbol<false>;
                plan->walk_smem = 256 + 64 * 8 + (size_t)kWarps * paired::kHeaderBytes;
                const int64_t slot_bytes = (int64_t)t.edge_cap * (int64_t)(sizeof(double4) + sizeof(int32_t)) + 4;
                plan->edge_chunk = std::max<int64_t>(4096, (int64_t)(4ull << 30) / slot_bytes);
                plan->kernel_label = std::string("soap_paired_kernel<1, 0, ") + (f64 ? "true" : "false") +
                                     ", 4, walk> + " + sv.name + " (edge lists)";
            }
        }
        if (plan->center_smem > budget1 || plan->structure_smem > budget1)
            return fail(MDSOAP_INVALID_ARGUMENT, "SOAP parameters need more shared memory than the device offers");
        *plan_out = plan.release();
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

void mdsoap_plan_destroy(mdsoap_plan* plan) { delete plan; }

int64_t mdsoap_plan_feature_count(const mdsoap_plan* plan) { return plan ? plan->features : 0; }

int64_t mdsoap_plan_rows(const mdsoap_plan* plan, const mdsoap_batch* batch) {
    if (!plan || !batch) return 0;
    return plan->average == MDSOAP_AVERAGE_OFF ? batch->atoms : batch->structures;
}

int mdsoap_compute(mdsoap_plan* plan, const mdsoap_batch* batch, void* out, const int32_t* devices,
                   int32_t n_devices, mdsoap_cancel_fn cancel, void* cancel_context) {
    if (!plan || !batch) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    try {
        validate_host_batch(plan, *batch);
        const int64_t rows = mdsoap_plan_rows(plan, batch);
        if (rows > 0 && !out) return fail(MDSOAP_INVALID_ARGUMENT, "null output buffer");
        if (cancel && cancel(cancel_context)) return fail(MDSOAP_CANCELLED, "descriptor computation was cancelled");
        std::vector<int> ids;
        if (devices && n_devices > 0)
            ids.assign(devices, devices + n_devices);
        else
            ids.push_back(0);
        if (batch->structures == 0 || rows == 0) {
            // Still resolve the device so a missing GPU fails loudly.
            plan->state(ids[0]);
            return MDSOAP_OK;
        }
        // Contiguous structure shards balanced by atom count.
        const int64_t S = batch->structures;
        const int parts = (int)std::min<int64_t>((int64_t)ids.size(), S);
        std::vector<int64_t> cuts{0};
        for (int i = 1; i < parts; ++i) {
            const int64_t goal = batch->atoms * i / parts;
            int64_t s = std::upper_bound(batch->offsets, batch->offsets + S + 1, goal) - batch->offsets - 1;
            s = std::max<int64_t>(s, cuts.back() + 1);
            s = std::min<int64_t>(s, S - (parts - i));
            cuts.push_back(s);
        }
        cuts.push_back(S);
        std::atomic<bool> stop{false};
        const size_t row_bytes = (size_t)plan->features * plan->out_elem();
        const bool by_structure = plan->average != MDSOAP_AVERAGE_OFF;
        std::vector<Failure> failures(parts);
        std::vector<bool> failed(parts, false);
        auto work = [&](int i) {
            try {
                const int64_t row0 = by_structure ? cuts[i] : batch->offsets[cuts[i]];
                plan->shard_compute(ids[i], *batch, cuts[i], cuts[i + 1], static_cast<char*>(out) + row0 * row_bytes,
                                    cancel, cancel_context, stop);
            } catch (const Failure& f) {
                failures[i] = f;
                failed[i] = true;
                stop.store(true);
            } catch (const std::exception& e) {
                failures[i] = Failure{MDSOAP_INTERNAL, e.what()};
                failed[i] = true;
                stop.store(true);
            }
        };
        if (parts == 1) {
            work(0);
        } else {
            std::vector<std::thread> threads;
            for (int i = 0; i < parts; ++i) threads.emplace_back(work, i);
            for (auto& t : threads) t.join();
        }
        // Report the first real failure ahead of secondary cancellations.
        for (int i = 0; i < parts; ++i)
            if (failed[i] && failures[i].status != MDSOAP_CANCELLED) return fail(failures[i].status, failures[i].message);
        for (int i = 0; i < parts; ++i)
            if (failed[i]) return fail(failures[i].status, failures[i].message);
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

int mdsoap_compute_device(mdsoap_plan* plan, const mdsoap_batch* batch, void* out, int32_t device, void* stream) {
    if (!plan || !batch) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    if (batch->structures < 0 || batch->atoms < 0) return fail(MDSOAP_INVALID_ARGUMENT, "invalid structure batch");
    try {
        DeviceState& st = plan->state(device);
        std::lock_guard<std::mutex> lock(st.mutex);
        check(cudaSetDevice(device), "cudaSetDevice");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        DeviceBatch db{batch->numbers, batch->positions, batch->cells, batch->pbc, batch->offsets, batch->structures,
                       batch->atoms};
        unsigned* error = st.error.as<unsigned>();
        const bool timed = plan->timing;
        if (timed && !st.timing[0])
            for (auto& e : st.timing) check(cudaEventCreate(&e), "timing event");
        if (timed) check(cudaEventRecord(st.timing[0], s), "timing event");
        plan->bin(st, db, s, error);
        if (timed) check(cudaEventRecord(st.timing[1], s), "timing event");
        // Structure ranges are only needed for the averages; the device batch
        // is one block.
        st.split_marks = 0;
        plan->run_block(st, db, 0, batch->structures, 0, batch->atoms, out, s, error, timed ? st.timing[2] : nullptr,
                        timed);
        if (timed) check(cudaEventRecord(st.timing[3], s), "timing event");
        st.timed = timed;
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

int mdsoap_plan_check(mdsoap_plan* plan, int32_t device, void* stream) {
    if (!plan) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    try {
        DeviceState& st = plan->state(device);
        check(cudaSetDevice(device), "cudaSetDevice");
        check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "stream sync");
        unsigned bits = 0;
        check(cudaMemcpy(&bits, st.error.ptr, sizeof(unsigned), cudaMemcpyDeviceToHost), "read error word");
        check(cudaMemset(st.error.ptr, 0, sizeof(unsigned)), "clear error word");
        if (bits)
            return fail(bits & (kErrUnknownSpecies | kErrMixedPbc | kErrSingularCell) ? MDSOAP_INVALID_ARGUMENT
                                                                                      : MDSOAP_INTERNAL,
                        device_error_text(bits));
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    }
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Sparse (CSR) rows.

struct mdsoap_csr {
    int64_t rows = 0, cols = 0, nnz = 0;
    int32_t dtype = MDSOAP_FLOAT32;
    std::vector<int64_t> indptr;
    std::vector<int32_t> indices;
    std::vector<unsigned char> data;
};

namespace {
// Device bytes freed when the call ends.
struct ScopedBytes : DeviceBytes {
    ScopedBytes() = default;
    ScopedBytes(const ScopedBytes&) = delete;
    ScopedBytes& operator=(const ScopedBytes&) = delete;
    ~ScopedBytes() { release(); }
};

template <class T>
void csr_from_device_rows(mdsoap_plan* plan, const void* dense, int64_t rows, int64_t cols, cudaStream_t s,
                          mdsoap_csr& csr) {
    ScopedBytes counts, indptr, indices, data;
    counts.reserve(8 * (size_t)rows, "CSR row counts");
    const unsigned grid = (unsigned)std::min<int64_t>((rows + kWarps - 1) / kWarps, 65535);
    csr_count_kernel<T><<<grid, kWarps * 32, 0, s>>>(static_cast<const T*>(dense), rows, cols, counts.as<int64_t>());
    check(cudaGetLastError(), "CSR count kernel launch");
    std::vector<int64_t> host_counts((size_t)rows);
    check(cudaMemcpyAsync(host_counts.data(), counts.ptr, 8 * (size_t)rows, cudaMemcpyDeviceToHost, s),
          "CSR row counts D2H");
    check(cudaStreamSynchronize(s), "stream sync");
    csr.indptr.assign((size_t)rows + 1, 0);
    for (int64_t r = 0; r < rows; ++r) csr.indptr[(size_t)r + 1] = csr.indptr[(size_t)r] + host_counts[(size_t)r];
    csr.nnz = csr.indptr[(size_t)rows];
    csr.indices.resize((size_t)csr.nnz);
    csr.data.resize((size_t)csr.nnz * sizeof(T));
    if (csr.nnz > 0) {
        indptr.reserve(8 * ((size_t)rows + 1), "CSR row offsets");
        indices.reserve(4 * (size_t)csr.nnz, "CSR column indices");
        data.reserve(sizeof(T) * (size_t)csr.nnz, "CSR values");
        check(cudaMemcpyAsync(indptr.ptr, csr.indptr.data(), 8 * ((size_t)rows + 1), cudaMemcpyHostToDevice, s),
              "CSR row offsets H2D");
        csr_fill_kernel<T><<<grid, kWarps * 32, 0, s>>>(static_cast<const T*>(dense), rows, cols,
                                                         indptr.as<int64_t>(), indices.as<int32_t>(), data.as<T>());
        check(cudaGetLastError(), "CSR fill kernel launch");
        check(cudaMemcpyAsync(csr.indices.data(), indices.ptr, 4 * (size_t)csr.nnz, cudaMemcpyDeviceToHost, s),
              "CSR indices D2H");
        check(cudaMemcpyAsync(csr.data.data(), data.ptr, sizeof(T) * (size_t)csr.nnz, cudaMemcpyDeviceToHost, s),
              "CSR values D2H");
        check(cudaStreamSynchronize(s), "stream sync");
        plan->launches.fetch_add(1, std::memory_order_relaxed);
    }
    plan->launches.fetch_add(1, std::memory_order_relaxed);
}
}  // namespace

extern "C" {

int mdsoap_compute_csr(mdsoap_plan* plan, const mdsoap_batch* batch, int32_t device, mdsoap_csr** csr_out) {
    if (!plan || !batch || !csr_out) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    *csr_out = nullptr;
    try {
        validate_host_batch(plan, *batch);
        auto csr = std::make_unique<mdsoap_csr>();
        const int64_t rows = mdsoap_plan_rows(plan, batch), cols = plan->features;
        csr->rows = rows;
        csr->cols = cols;
        csr->dtype = plan->out_dtype;
        csr->indptr.assign((size_t)rows + 1, 0);
        DeviceState& st = plan->state(device);
        if (batch->structures == 0 || rows == 0) {
            *csr_out = csr.release();
            return MDSOAP_OK;
        }
        std::lock_guard<std::mutex> lock(st.mutex);
        check(cudaSetDevice(device), "cudaSetDevice");
        cudaStream_t s = st.compute;
        const int64_t S = batch->structures, N = batch->atoms;
        ScopedBytes numbers, positions, cells, pbc, offsets, dense;
        numbers.reserve(4 * (size_t)N, "batch numbers");
        positions.reserve(24 * (size_t)N, "batch positions");
        cells.reserve(72 * (size_t)S, "batch cells");
        pbc.reserve(12 * (size_t)S, "batch pbc");
        offsets.reserve(8 * ((size_t)S + 1), "batch offsets");
        dense.reserve((size_t)rows * (size_t)cols * plan->out_elem(), "dense rows");
        check(cudaMemcpyAsync(numbers.ptr, batch->numbers, 4 * (size_t)N, cudaMemcpyHostToDevice, s), "H2D numbers");
        check(cudaMemcpyAsync(positions.ptr, batch->positions, 24 * (size_t)N, cudaMemcpyHostToDevice, s),
              "H2D positions");
        check(cudaMemcpyAsync(cells.ptr, batch->cells, 72 * (size_t)S, cudaMemcpyHostToDevice, s), "H2D cells");
        check(cudaMemcpyAsync(pbc.ptr, batch->pbc, 12 * (size_t)S, cudaMemcpyHostToDevice, s), "H2D pbc");
        check(cudaMemcpyAsync(offsets.ptr, batch->offsets, 8 * ((size_t)S + 1), cudaMemcpyHostToDevice, s),
              "H2D offsets");
        DeviceBatch db{numbers.as<int32_t>(), positions.as<double>(), cells.as<double>(), pbc.as<int32_t>(),
                       offsets.as<int64_t>(), S, N};
        unsigned* error = st.error.as<unsigned>();
        plan->bin(st, db, s, error);
        plan->run_block(st, db, 0, S, 0, N, dense.ptr, s, error);
        unsigned bits = 0;
        check(cudaMemcpyAsync(&bits, error, sizeof(unsigned), cudaMemcpyDeviceToHost, s), "read error word");
        check(cudaStreamSynchronize(s), "stream sync");
        if (bits) {
            check(cudaMemset(error, 0, sizeof(unsigned)), "clear error word");
            return fail(bits & (kErrUnknownSpecies | kErrMixedPbc | kErrSingularCell) ? MDSOAP_INVALID_ARGUMENT
                                                                                      : MDSOAP_INTERNAL,
                        device_error_text(bits));
        }
        if (plan->out_dtype == MDSOAP_FLOAT64)
            csr_from_device_rows<double>(plan, dense.ptr, rows, cols, s, *csr);
        else
            csr_from_device_rows<float>(plan, dense.ptr, rows, cols, s, *csr);
        *csr_out = csr.release();
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

int mdsoap_csr_info(const mdsoap_csr* csr, int64_t* rows, int64_t* cols, int64_t* nnz) {
    if (!csr) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    if (rows) *rows = csr->rows;
    if (cols) *cols = csr->cols;
    if (nnz) *nnz = csr->nnz;
    return MDSOAP_OK;
}

int mdsoap_csr_copy(const mdsoap_csr* csr, int64_t* indptr, int32_t* indices, void* data) {
    if (!csr || !indptr || ((!indices || !data) && csr->nnz > 0)) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    std::memcpy(indptr, csr->indptr.data(), 8 * csr->indptr.size());
    if (csr->nnz > 0) {
        std::memcpy(indices, csr->indices.data(), 4 * (size_t)csr->nnz);
        std::memcpy(data, csr->data.data(), csr->data.size());
    }
    return MDSOAP_OK;
}

void mdsoap_csr_destroy(mdsoap_csr* csr) { delete csr; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free device entry point.  The scratch array below is the only
// device memory it uses; its host-side name is only a stand-in, so the device
// address is looked up once per device with cudaGetSymbolAddress.

__device__ __align__(256) unsigned char g_noalloc_scratch[MDSOAP_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_noalloc_mutex;
unsigned char* g_noalloc_base[64] = {};  // device address of the array, per device ordinal

unsigned char* noalloc_base(int device) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (device < 0 || device >= 64) raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device index out of range");
    if (g_noalloc_base[device]) return g_noalloc_base[device];
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    check(err, "cudaGetSymbolAddress(no-allocation scratch)");
    g_noalloc_base[device] = static_cast<unsigned char*>(ptr);
    return g_noalloc_base[device];
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

extern "C" {

int mdsoap_compute_device_noalloc(mdsoap_plan* plan, const mdsoap_batch* batch, void* out, int32_t device,
                                  void* stream) {
    if (!plan || !batch) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    if (batch->structures < 0 || batch->atoms < 0) return fail(MDSOAP_INVALID_ARGUMENT, "invalid structure batch");
    try {
        const int64_t S = batch->structures, N = batch->atoms;
        // Scratch layout (each piece 256-byte aligned).
        size_t off = 0;
        auto take = [&](size_t bytes) {
            const size_t at = off;
            off = align256(off + std::max<size_t>(bytes, 1));
            return at;
        };
        const size_t o_items = take(sizeof(RadialItem) * plan->items.size());
        const size_t o_betas = take(8 * plan->betas.size());
        const size_t o_species = take(4 * plan->species.size());
        const size_t o_poly = take(8 * plan->poly.size());
        const size_t o_error = take(sizeof(unsigned));
        const size_t o_info = take(sizeof(StructInfo) * (size_t)std::max<int64_t>(S, 1));
        const size_t o_struct = take(4 * (size_t)N);
        const size_t o_type = take(4 * (size_t)N);
        const size_t o_bin = take(4 * (size_t)N);
        const size_t o_wrap = take(12 * (size_t)N);
        const size_t o_sorted = take(4 * (size_t)N);
        const size_t o_spos = take(32 * (size_t)N);
        const size_t bins = (size_t)(2 * N + 8 * S + 8);
        const size_t o_bstart = take(4 * bins);
        const size_t o_bcursor = take(4 * bins);
        size_t o_cbuf = 0, o_pbuf = 0, o_rbuf = 0;
        if (plan->average == MDSOAP_AVERAGE_INNER) o_cbuf = take(8 * (size_t)N * (size_t)plan->csize);
        if (plan->average == MDSOAP_AVERAGE_OUTER) o_pbuf = take(8 * (size_t)N * (size_t)plan->features);
        if (plan->tab.r_global) o_rbuf = take(8 * (size_t)N * (size_t)plan->tab.rsize);
        if (off > MDSOAP_NOALLOC_SCRATCH_BYTES)
            return fail(MDSOAP_CAPACITY_OVERFLOW,
                        "batch needs " + std::to_string(off) + " bytes of scratch; the no-allocation entry point holds " +
                            std::to_string((size_t)MDSOAP_NOALLOC_SCRATCH_BYTES) + " bytes (split the batch)");
        if (N > 2147483647LL) return fail(MDSOAP_INVALID_ARGUMENT, "neighbor atom index exceeds int32 range");
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
            cudaGetLastError();
            raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device unavailable");
        }
        check(cudaSetDevice(device), "cudaSetDevice");
        unsigned char* base = noalloc_base(device);
        int optin = 0;
        check(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device), "smem attribute");
        if (plan->center_smem > (size_t)optin || plan->structure_smem > (size_t)optin)
            raise(MDSOAP_INVALID_ARGUMENT, "SOAP parameters need more shared memory than the device offers");
        check(cudaFuncSetAttribute(plan->variant->center_sym(), cudaFuncAttributeMaxDynamicSharedMemorySize, optin),
              "center kernel smem");
        check(cudaFuncSetAttribute(plan->variant->structure_sym(), cudaFuncAttributeMaxDynamicSharedMemorySize, optin),
              "structure kernel smem");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        // Plan tables (the array keeps the previous call's contents: refresh them).
        check(cudaMemcpyAsync(base + o_items, plan->items.data(), sizeof(RadialItem) * plan->items.size(),
                              cudaMemcpyHostToDevice, st),
              "upload radial items");
        check(cudaMemcpyAsync(base + o_betas, plan->betas.data(), 8 * plan->betas.size(), cudaMemcpyHostToDevice, st),
              "upload betas");
        check(cudaMemcpyAsync(base + o_species, plan->species.data(), 4 * plan->species.size(),
                              cudaMemcpyHostToDevice, st),
              "upload species");
        if (!plan->poly.empty())
            check(cudaMemcpyAsync(base + o_poly, plan->poly.data(), 8 * plan->poly.size(), cudaMemcpyHostToDevice, st),
                  "upload polynomial basis");
        unsigned* error = reinterpret_cast<unsigned*>(base + o_error);
        check(cudaMemsetAsync(error, 0, sizeof(unsigned), st), "clear error word");
        BinView v;
        v.info = reinterpret_cast<StructInfo*>(base + o_info);
        v.struct_of = reinterpret_cast<int32_t*>(base + o_struct);
        v.type = reinterpret_cast<int32_t*>(base + o_type);
        v.bin_of = reinterpret_cast<int32_t*>(base + o_bin);
        v.wrap = reinterpret_cast<int32_t*>(base + o_wrap);
        v.sorted = reinterpret_cast<int32_t*>(base + o_sorted);
        v.bin_start = reinterpret_cast<int32_t*>(base + o_bstart);
        v.bin_cursor = reinterpret_cast<int32_t*>(base + o_bcursor);
        v.error = error;
        v.spos = reinterpret_cast<double4*>(base + o_spos);
        DeviceBatch db{batch->numbers, batch->positions, batch->cells, batch->pbc, batch->offsets, S, N};
        if (S > 0) {
            bin_structures_kernel<<<(unsigned)S, 256, 0, st>>>(db, v, plan->cutoff,
                                                               reinterpret_cast<int32_t*>(base + o_species),
                                                               plan->n_species);
            check(cudaGetLastError(), "bin kernel launch");
            plan->launches.fetch_add(1, std::memory_order_relaxed);
        }
        SoapPointers p{};
        p.positions = db.positions;
        p.bins = v;
        p.items = reinterpret_cast<RadialItem*>(base + o_items);
        p.betas = reinterpret_cast<double*>(base + o_betas);
        p.poly = reinterpret_cast<double*>(base + o_poly);
        p.out = out;
        p.cbuf = o_cbuf ? reinterpret_cast<double*>(base + o_cbuf) : nullptr;
        p.pbuf = o_pbuf ? reinterpret_cast<double*>(base + o_pbuf) : nullptr;
        p.rbuf = o_rbuf ? reinterpret_cast<double*>(base + o_rbuf) : nullptr;
        p.out_row_begin = 0;
        p.center_begin = 0;
        p.center_end = N;
        p.grid_begin = 0;
        p.grid_end = N;
        if (N > 0) {
            // One launch with the tail fused in (no scratch for a split tail here).
            SoapTables fused = plan->tab;
            fused.split_tail = 0;
            const int64_t grid = (N + kWarps - 1) / kWarps;
            plan->variant->center(dim3((unsigned)grid), plan->center_smem, st, fused, p);
            check(cudaGetLastError(), "centre kernel launch");
            plan->launches.fetch_add(1, std::memory_order_relaxed);
        }
        if (plan->average != MDSOAP_AVERAGE_OFF && S > 0) {
            plan->variant->structure(dim3((unsigned)S), plan->structure_smem, st, plan->tab, db.offsets, 0, S, p.cbuf,
                                     p.pbuf, out, 0);
            check(cudaGetLastError(), "structure kernel launch");
            plan->launches.fetch_add(1, std::memory_order_relaxed);
        }
        unsigned bits = 0;
        check(cudaMemcpyAsync(&bits, error, sizeof(unsigned), cudaMemcpyDeviceToHost, st), "read error word");
        check(cudaStreamSynchronize(st), "stream sync");
        if (bits)
            return fail(bits & (kErrUnknownSpecies | kErrMixedPbc | kErrSingularCell) ? MDSOAP_INVALID_ARGUMENT
                                                                                      : MDSOAP_INTERNAL,
                        device_error_text(bits));
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

int mdsoap_plan_set_timing(mdsoap_plan* plan, int32_t enable) {
    if (!plan) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    plan->timing = enable != 0;
    return MDSOAP_OK;
}

int mdsoap_plan_last_timing(mdsoap_plan* plan, int32_t device, double* bin_ms, double* center_ms,
                            double* structure_ms) {
    if (!plan) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    try {
        DeviceState& st = plan->state(device);
        if (!st.timed) return fail(MDSOAP_INVALID_ARGUMENT, "no timed device call on this device");
        check(cudaSetDevice(device), "cudaSetDevice");
        check(cudaEventSynchronize(st.timing[3]), "timing sync");
        float a = 0, b = 0, c = 0;
        check(cudaEventElapsedTime(&a, st.timing[0], st.timing[1]), "elapsed");
        check(cudaEventElapsedTime(&b, st.timing[1], st.timing[2]), "elapsed");
        check(cudaEventElapsedTime(&c, st.timing[2], st.timing[3]), "elapsed");
        if (bin_ms) *bin_ms = a;
        if (center_ms) *center_ms = b;
        if (structure_ms) *structure_ms = c;
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    }
}

const char* mdsoap_plan_kernel(const mdsoap_plan* plan) {
    if (!plan || !plan->variant) return "";
    return plan->kernel_label.empty() ? plan->variant->name : plan->kernel_label.c_str();
}

int mdsoap_plan_last_timing_split(mdsoap_plan* plan, int32_t device, double* expansion_ms, double* tail_ms) {
    if (!plan) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    try {
        DeviceState& st = plan->state(device);
        if (!st.timed) return fail(MDSOAP_INVALID_ARGUMENT, "no timed device call on this device");
        check(cudaSetDevice(device), "cudaSetDevice");
        check(cudaEventSynchronize(st.timing[3]), "timing sync");
        double a = 0, b = 0;
        if (st.split_marks >= 2) {
            // Chunk i: expansion from the previous mark (the centre-phase start
            // for the first chunk) to marks[2i], tail from marks[2i] to marks[2i+1].
            cudaEvent_t prev = st.timing[1];
            for (size_t i = 0; i + 1 < st.split_marks; i += 2) {
                float x = 0, y = 0;
                check(cudaEventElapsedTime(&x, prev, st.marks[i]), "elapsed");
                check(cudaEventElapsedTime(&y, st.marks[i], st.marks[i + 1]), "elapsed");
                a += x;
                b += y;
                prev = st.marks[i + 1];
            }
        } else {
            float x = 0;
            check(cudaEventElapsedTime(&x, st.timing[1], st.timing[2]), "elapsed");
            a = x;
        }
        if (expansion_ms) *expansion_ms = a;
        if (tail_ms) *tail_ms = b;
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    }
}

int mdsoap_plan_launch_count(const mdsoap_plan* plan, int64_t* count) {
    if (!plan || !count) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    *count = plan->launches.load(std::memory_order_relaxed);
    return MDSOAP_OK;
}

int mdsoap_probe_exp(int32_t device, const double* x, int64_t count, double* ours, double* cuda_exp) {
    if (count < 0 || (count > 0 && (!x || !ours || !cuda_exp))) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    try {
        int devices = 0;
        if (cudaGetDeviceCount(&devices) != cudaSuccess || device < 0 || device >= devices)
            raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device unavailable");
        check(cudaSetDevice(device), "cudaSetDevice");
        if (count == 0) return MDSOAP_OK;
        DeviceBytes dx, d1, d2;
        const size_t bytes = 8 * (size_t)count;
        dx.reserve(bytes, "probe input");
        d1.reserve(bytes, "probe output");
        d2.reserve(bytes, "probe output");
        check(cudaMemcpy(dx.ptr, x, bytes, cudaMemcpyHostToDevice), "probe upload");
        exp_probe_kernel<<<256, 256>>>(dx.as<double>(), count, d1.as<double>(), d2.as<double>());
        check(cudaGetLastError(), "probe launch");
        check(cudaMemcpy(ours, d1.ptr, bytes, cudaMemcpyDeviceToHost), "probe download");
        check(cudaMemcpy(cuda_exp, d2.ptr, bytes, cudaMemcpyDeviceToHost), "probe download");
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    }
}

int mdsoap_probe_radial(int32_t device, int32_t form, const double* u, const double* e, const double* pref,
                        int64_t count, double* ours, double* cuda_exp) {
    if (form < 0 || form > 2) return fail(MDSOAP_INVALID_ARGUMENT, "form must be 0, 1 or 2");
    if (count < 0 || (count > 0 && (!u || !e || !pref || !ours || !cuda_exp)))
        return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    try {
        int devices = 0;
        if (cudaGetDeviceCount(&devices) != cudaSuccess || device < 0 || device >= devices)
            raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device unavailable");
        check(cudaSetDevice(device), "cudaSetDevice");
        if (count == 0) return MDSOAP_OK;
        DeviceBytes du, de, dp, d1, d2;
        const size_t bytes = 8 * (size_t)count;
        du.reserve(bytes, "probe input");
        de.reserve(bytes, "probe input");
        dp.reserve(bytes, "probe input");
        d1.reserve(bytes, "probe output");
        d2.reserve(bytes, "probe output");
        check(cudaMemcpy(du.ptr, u, bytes, cudaMemcpyHostToDevice), "probe upload");
        check(cudaMemcpy(de.ptr, e, bytes, cudaMemcpyHostToDevice), "probe upload");
        check(cudaMemcpy(dp.ptr, pref, bytes, cudaMemcpyHostToDevice), "probe upload");
        radial_probe_kernel<<<256, 256>>>(form, du.as<double>(), de.as<double>(), dp.as<double>(), count,
                                          d1.as<double>(), d2.as<double>());
        check(cudaGetLastError(), "probe launch");
        check(cudaMemcpy(ours, d1.ptr, bytes, cudaMemcpyDeviceToHost), "probe download");
        check(cudaMemcpy(cuda_exp, d2.ptr, bytes, cudaMemcpyDeviceToHost), "probe download");
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& ex) {
        return fail(MDSOAP_INTERNAL, ex.what());
    }
}

int mdsoap_probe_bounded_wait(int32_t device, uint64_t limit_ns) {
    if (limit_ns == 0 || limit_ns > 2000000000ull)
        return fail(MDSOAP_INVALID_ARGUMENT, "limit_ns must be in (0, 2 s]");
    try {
        int devices = 0;
        if (cudaGetDeviceCount(&devices) != cudaSuccess || device < 0 || device >= devices)
            raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device unavailable");
        check(cudaSetDevice(device), "cudaSetDevice");
        DeviceBytes word;
        word.reserve(sizeof(unsigned), "error word");
        check(cudaMemset(word.ptr, 0, sizeof(unsigned)), "clear error word");
        bounded_wait_probe_kernel<<<1, 32>>>(word.as<unsigned>(), limit_ns);
        check(cudaGetLastError(), "probe launch");
        unsigned bits = 0;
        check(cudaMemcpy(&bits, word.ptr, sizeof(unsigned), cudaMemcpyDeviceToHost), "read error word");
        if (bits)
            return fail(bits & (kErrUnknownSpecies | kErrMixedPbc | kErrSingularCell) ? MDSOAP_INVALID_ARGUMENT
                                                                                      : MDSOAP_INTERNAL,
                        device_error_text(bits));
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

namespace {

// Idle page-locked result buffers, by capacity.  Never destroyed: unlocking
// memory after the CUDA runtime has shut down at process exit is not allowed.
struct HostPool {
    std::mutex mutex;
    std::multimap<size_t, void*> idle;           // capacity -> buffer
    std::unordered_map<void*, size_t> capacity;  // every buffer handed out or idle
    size_t idle_bytes = 0;
};

HostPool& host_pool() {
    static HostPool* pool = new HostPool();
    return *pool;
}

size_t host_pool_limit() {
    const char* env = std::getenv("MDSOAP_HOST_POOL_BYTES");
    return env ? (size_t)std::strtoull(env, nullptr, 10) : ((size_t)4 << 30);
}

}  // namespace

int mdsoap_host_buffer_acquire(size_t bytes, void** ptr) {
    if (!ptr) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    *ptr = nullptr;
    try {
        HostPool& pool = host_pool();
        const size_t want = std::max<size_t>(bytes, 1);
        {
            std::lock_guard<std::mutex> lock(pool.mutex);
            auto it = pool.idle.lower_bound(want);
            if (it != pool.idle.end() && it->first <= 2 * want) {
                *ptr = it->second;
                pool.idle_bytes -= it->first;
                pool.idle.erase(it);
                return MDSOAP_OK;
            }
        }
        // Capacity rounded up to 2 MiB so that nearby sizes share buffers.
        const size_t cap = (want + ((size_t)2 << 20) - 1) & ~(((size_t)2 << 20) - 1);
        void* p = nullptr;
        const cudaError_t err = cudaMallocHost(&p, cap);
        if (err != cudaSuccess) {
            cudaGetLastError();
            return fail(MDSOAP_OUT_OF_MEMORY, std::string("page-locked result buffer: ") + cudaGetErrorString(err));
        }
        std::lock_guard<std::mutex> lock(pool.mutex);
        pool.capacity[p] = cap;
        *ptr = p;
        return MDSOAP_OK;
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

void mdsoap_host_buffer_release(void* ptr) {
    if (!ptr) return;
    HostPool& pool = host_pool();
    void* unlock = nullptr;
    {
        std::lock_guard<std::mutex> lock(pool.mutex);
        auto it = pool.capacity.find(ptr);
        if (it == pool.capacity.end()) return;  // not ours
        const size_t cap = it->second;
        if (pool.idle_bytes + cap <= host_pool_limit()) {
            pool.idle.emplace(cap, ptr);
            pool.idle_bytes += cap;
        } else {
            pool.capacity.erase(it);
            unlock = ptr;
        }
    }
    if (unlock) cudaFreeHost(unlock);
}

int mdsoap_probe_fp64_fma(int32_t device, double* tflops) {
    if (!tflops) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    try {
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
            raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device unavailable");
        check(cudaSetDevice(device), "cudaSetDevice");
        int sms = 0;
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "SM count");
        DeviceBytes sink;
        const int blocks = sms * 8, threads = 256;
        sink.reserve(8 * (size_t)blocks * threads, "probe sink");
        cudaEvent_t e0, e1;
        check(cudaEventCreate(&e0), "event");
        check(cudaEventCreate(&e1), "event");
        const int iters = 4096;
        fma_probe_kernel<<<blocks, threads>>>(sink.as<double>(), iters);  // warm-up
        check(cudaEventRecord(e0), "event");
        const int reps = 8;
        for (int r = 0; r < reps; ++r) fma_probe_kernel<<<blocks, threads>>>(sink.as<double>(), iters);
        check(cudaEventRecord(e1), "event");
        check(cudaEventSynchronize(e1), "probe sync");
        float ms = 0;
        check(cudaEventElapsedTime(&ms, e0, e1), "elapsed");
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        sink.release();
        const double flops = 2.0 * kProbeChains * (double)iters * blocks * threads * reps;
        *tflops = flops / (ms * 1e-3) / 1e12;
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    }
}

int mdsoap_graph_build(const mdsoap_batch* batch, double cutoff, int32_t device, mdsoap_graph** graph_out) {
    if (!batch || !graph_out) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    *graph_out = nullptr;
    if (!std::isfinite(cutoff) || cutoff <= 0.0)
        return fail(MDSOAP_INVALID_ARGUMENT, "neighbor cutoff must be finite and positive");
    try {
        validate_host_batch(nullptr, *batch);
        int count = 0;
        const cudaError_t probe_err = cudaGetDeviceCount(&count);
        if (probe_err != cudaSuccess || count == 0)
            raise(MDSOAP_DEVICE_UNAVAILABLE, std::string("no CUDA device available: ") + cudaGetErrorString(probe_err));
        if (device < 0 || device >= count) raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device index out of range");
        check(cudaSetDevice(device), "cudaSetDevice");
        auto g = std::make_unique<mdsoap_graph>();
        const int64_t atoms = batch->atoms, S = batch->structures;
        g->atoms = atoms;
        g->offsets.assign(atoms + 1, 0);
        if (atoms == 0 || S == 0) {
            *graph_out = g.release();
            return MDSOAP_OK;
        }
        cudaStream_t stream = nullptr;
        check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
        struct StreamGuard {
            cudaStream_t s;
            ~StreamGuard() { cudaStreamDestroy(s); }
        } guard{stream};
        Workspace w;
        struct WorkGuard {
            Workspace& w;
            ~WorkGuard() { w.release(); }
        } wguard{w};
        DeviceBytes error, counts, offsets_d, atoms_d, shifts_d, disp_d, d2_d;
        struct BytesGuard {
            std::vector<DeviceBytes*> list;
            ~BytesGuard() {
                for (auto* b : list) b->release();
            }
        } bguard{{&error, &counts, &offsets_d, &atoms_d, &shifts_d, &disp_d, &d2_d}};
        w.numbers.reserve(4 * atoms, "numbers");
        w.positions.reserve(24 * atoms, "positions");
        w.cells.reserve(72 * S, "cells");
        w.pbc.reserve(12 * S, "pbc");
        w.offsets.reserve(8 * (S + 1), "offsets");
        check(cudaMemcpyAsync(w.numbers.ptr, batch->numbers, 4 * atoms, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.positions.ptr, batch->positions, 24 * atoms, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.cells.ptr, batch->cells, 72 * S, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.pbc.ptr, batch->pbc, 12 * S, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.offsets.ptr, batch->offsets, 8 * (S + 1), cudaMemcpyHostToDevice, stream), "H2D");
        error.reserve(64, "error");
        check(cudaMemsetAsync(error.ptr, 0, 64, stream), "memset");
        w.reserve_bins(atoms, S);
        DeviceBatch db{w.numbers.as<int32_t>(), w.positions.as<double>(), w.cells.as<double>(), w.pbc.as<int32_t>(),
                       w.offsets.as<int64_t>(), S, atoms};
        // Species lookup is irrelevant here: pass an empty list (types -> -1,
        // the unknown-species bit is ignored below).
        bin_structures_kernel<<<(unsigned)S, 256, 0, stream>>>(db, w.bins(error.as<unsigned>()), cutoff, nullptr, 0);
        check(cudaGetLastError(), "bin kernel");
        counts.reserve(8 * atoms, "counts");
        const double cutoff2 = cutoff * cutoff;
        const unsigned grid = (unsigned)((atoms + 7) / 8);
        graph_count_kernel<<<grid, 256, 0, stream>>>(db.positions, w.bins(error.as<unsigned>()), atoms, cutoff2,
                                                     counts.as<int64_t>());
        check(cudaGetLastError(), "count kernel");
        std::vector<int64_t> host_counts(atoms);
        check(cudaMemcpyAsync(host_counts.data(), counts.ptr, 8 * atoms, cudaMemcpyDeviceToHost, stream), "D2H counts");
        check(cudaStreamSynchronize(stream), "sync");
        unsigned bits = 0;
        check(cudaMemcpy(&bits, error.ptr, sizeof(unsigned), cudaMemcpyDeviceToHost), "error word");
        bits &= ~kErrUnknownSpecies;
        if (bits) raise(bits & (kErrMixedPbc | kErrSingularCell) ? MDSOAP_INVALID_ARGUMENT : MDSOAP_INTERNAL,
                        device_error_text(bits));
        for (int64_t a = 0; a < atoms; ++a) g->offsets[a + 1] = g->offsets[a] + host_counts[a];
        const int64_t pairs = g->offsets[atoms];
        offsets_d.reserve(8 * (atoms + 1), "offsets");
        atoms_d.reserve(4 * std::max<int64_t>(pairs, 1), "pair atoms");
        shifts_d.reserve(12 * std::max<int64_t>(pairs, 1), "pair shifts");
        disp_d.reserve(24 * std::max<int64_t>(pairs, 1), "pair displacements");
        d2_d.reserve(8 * std::max<int64_t>(pairs, 1), "pair distances");
        check(cudaMemcpyAsync(offsets_d.ptr, g->offsets.data(), 8 * (atoms + 1), cudaMemcpyHostToDevice, stream), "H2D");
        graph_fill_kernel<<<grid, 256, 0, stream>>>(db.positions, w.bins(error.as<unsigned>()), atoms, cutoff2,
                                                    offsets_d.as<int64_t>(), atoms_d.as<int32_t>(),
                                                    shifts_d.as<int32_t>(), disp_d.as<double>(), d2_d.as<double>());
        check(cudaGetLastError(), "fill kernel");
        g->atom_ids.resize(pairs);
        g->shifts.resize(3 * pairs);
        g->displacements.resize(3 * pairs);
        g->distance2.resize(pairs);
        if (pairs) {
            check(cudaMemcpyAsync(g->atom_ids.data(), atoms_d.ptr, 4 * pairs, cudaMemcpyDeviceToHost, stream), "D2H");
            check(cudaMemcpyAsync(g->shifts.data(), shifts_d.ptr, 12 * pairs, cudaMemcpyDeviceToHost, stream), "D2H");
            check(cudaMemcpyAsync(g->displacements.data(), disp_d.ptr, 24 * pairs, cudaMemcpyDeviceToHost, stream), "D2H");
            check(cudaMemcpyAsync(g->distance2.data(), d2_d.ptr, 8 * pairs, cudaMemcpyDeviceToHost, stream), "D2H");
        }
        check(cudaStreamSynchronize(stream), "sync");
        check(cudaMemcpy(&bits, error.ptr, sizeof(unsigned), cudaMemcpyDeviceToHost), "error word");
        bits &= ~kErrUnknownSpecies;
        if (bits) raise(MDSOAP_INTERNAL, device_error_text(bits));
        *graph_out = g.release();
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

int mdsoap_neighbor_list(const mdsoap_batch* batch, double cutoff, int32_t full_list, int32_t self_pairs,
                         int32_t device, mdsoap_pairs** pairs_out) {
    if (!batch || !pairs_out) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    *pairs_out = nullptr;
    if (!std::isfinite(cutoff) || cutoff <= 0.0)
        return fail(MDSOAP_INVALID_ARGUMENT, "neighbor cutoff must be finite and positive");
    try {
        validate_host_batch(nullptr, *batch);
        int count = 0;
        const cudaError_t probe_err = cudaGetDeviceCount(&count);
        if (probe_err != cudaSuccess || count == 0)
            raise(MDSOAP_DEVICE_UNAVAILABLE, std::string("no CUDA device available: ") + cudaGetErrorString(probe_err));
        if (device < 0 || device >= count) raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device index out of range");
        check(cudaSetDevice(device), "cudaSetDevice");
        auto out = std::make_unique<mdsoap_pairs>();
        const int64_t atoms = batch->atoms, S = batch->structures;
        out->row_offsets.assign(S + 1, 0);
        if (atoms == 0 || S == 0) {
            *pairs_out = out.release();
            return MDSOAP_OK;
        }
        cudaStream_t stream = nullptr;
        check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
        struct StreamGuard {
            cudaStream_t s;
            ~StreamGuard() { cudaStreamDestroy(s); }
        } guard{stream};
        Workspace w;
        struct WorkGuard {
            Workspace& w;
            ~WorkGuard() { w.release(); }
        } wguard{w};
        DeviceBytes error, counts, offsets_d, grids, records_d, values_d;
        struct BytesGuard {
            std::vector<DeviceBytes*> list;
            ~BytesGuard() {
                for (auto* b : list) b->release();
            }
        } bguard{{&error, &counts, &offsets_d, &grids, &records_d, &values_d}};
        w.numbers.reserve(4 * atoms, "numbers");
        w.positions.reserve(24 * atoms, "positions");
        w.cells.reserve(72 * S, "cells");
        w.pbc.reserve(12 * S, "pbc");
        w.offsets.reserve(8 * (S + 1), "offsets");
        check(cudaMemcpyAsync(w.numbers.ptr, batch->numbers, 4 * atoms, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.positions.ptr, batch->positions, 24 * atoms, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.cells.ptr, batch->cells, 72 * S, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.pbc.ptr, batch->pbc, 12 * S, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.offsets.ptr, batch->offsets, 8 * (S + 1), cudaMemcpyHostToDevice, stream), "H2D");
        error.reserve(64, "error");
        check(cudaMemsetAsync(error.ptr, 0, 64, stream), "memset");
        w.reserve_bins(atoms, S);
        DeviceBatch db{w.numbers.as<int32_t>(), w.positions.as<double>(), w.cells.as<double>(), w.pbc.as<int32_t>(),
                       w.offsets.as<int64_t>(), S, atoms};
        BinView bins = w.bins(error.as<unsigned>());
        bin_structures_kernel<<<(unsigned)S, 256, 0, stream>>>(db, bins, cutoff, nullptr, 0);
        check(cudaGetLastError(), "bin kernel");
        grids.reserve(sizeof(CanonGrid) * S, "neighbour list grids");
        canon_grid_kernel<<<(unsigned)S, 256, 0, stream>>>(db, bins, cutoff, grids.as<CanonGrid>());
        check(cudaGetLastError(), "grid kernel");
        counts.reserve(8 * atoms, "counts");
        const double cutoff2 = cutoff * cutoff;
        const unsigned grid = (unsigned)((atoms + kWarps - 1) / kWarps);
        list_count_kernel<<<grid, kWarps * 32, 0, stream>>>(db.positions, bins, atoms, cutoff2, full_list != 0,
                                                              self_pairs != 0, counts.as<int64_t>());
        check(cudaGetLastError(), "count kernel");
        std::vector<int64_t> host_counts(atoms);
        check(cudaMemcpyAsync(host_counts.data(), counts.ptr, 8 * atoms, cudaMemcpyDeviceToHost, stream), "D2H counts");
        check(cudaStreamSynchronize(stream), "sync");
        unsigned bits = 0;
        check(cudaMemcpy(&bits, error.ptr, sizeof(unsigned), cudaMemcpyDeviceToHost), "error word");
        bits &= ~kErrUnknownSpecies;
        if (bits) raise(bits & (kErrMixedPbc | kErrSingularCell) ? MDSOAP_INVALID_ARGUMENT : MDSOAP_INTERNAL,
                        device_error_text(bits));
        std::vector<int64_t> centre_rows(atoms + 1, 0);
        for (int64_t a = 0; a < atoms; ++a) centre_rows[a + 1] = centre_rows[a] + host_counts[a];
        for (int64_t s = 0; s <= S; ++s) out->row_offsets[s] = centre_rows[batch->offsets[s]];
        const int64_t pairs = centre_rows[atoms];
        out->records.resize(5 * pairs);
        out->values.resize(4 * pairs);
        if (pairs > 0) {
            offsets_d.reserve(8 * (atoms + 1), "row offsets");
            records_d.reserve(40 * pairs, "pair records");
            values_d.reserve(32 * pairs, "pair values");
            check(cudaMemcpyAsync(offsets_d.ptr, centre_rows.data(), 8 * (atoms + 1), cudaMemcpyHostToDevice, stream),
                  "H2D");
            const size_t smem = (size_t)kWarps * kListCapacity * sizeof(unsigned long long);
            check(cudaFuncSetAttribute(list_fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                  "list kernel smem");
            list_fill_kernel<<<grid, kWarps * 32, smem, stream>>>(db.positions, bins, grids.as<CanonGrid>(), atoms,
                                                                   cutoff2, full_list != 0, self_pairs != 0,
                                                                   offsets_d.as<int64_t>(), records_d.as<double>(),
                                                                   values_d.as<double>());
            check(cudaGetLastError(), "list kernel");
            check(cudaMemcpyAsync(out->records.data(), records_d.ptr, 40 * pairs, cudaMemcpyDeviceToHost, stream),
                  "D2H");
            check(cudaMemcpyAsync(out->values.data(), values_d.ptr, 32 * pairs, cudaMemcpyDeviceToHost, stream), "D2H");
        }
        check(cudaStreamSynchronize(stream), "sync");
        check(cudaMemcpy(&bits, error.ptr, sizeof(unsigned), cudaMemcpyDeviceToHost), "error word");
        bits &= ~kErrUnknownSpecies;
        if (bits) raise(bits & kErrPairCapacity ? MDSOAP_CAPACITY_OVERFLOW : MDSOAP_INTERNAL, device_error_text(bits));
        *pairs_out = out.release();
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

int64_t mdsoap_pairs_count(const mdsoap_pairs* pairs) { return pairs ? (int64_t)pairs->values.size() / 4 : 0; }

int mdsoap_pairs_copy(const mdsoap_pairs* pairs, double* records, double* values, int64_t* row_offsets) {
    if (!pairs) return fail(MDSOAP_INVALID_ARGUMENT, "null pair table");
    if (records && !pairs->records.empty())
        std::memcpy(records, pairs->records.data(), 8 * pairs->records.size());
    if (values && !pairs->values.empty()) std::memcpy(values, pairs->values.data(), 8 * pairs->values.size());
    if (row_offsets) std::memcpy(row_offsets, pairs->row_offsets.data(), 8 * pairs->row_offsets.size());
    return MDSOAP_OK;
}

void mdsoap_pairs_destroy(mdsoap_pairs* pairs) { delete pairs; }

int64_t mdsoap_graph_pairs(const mdsoap_graph* graph) { return graph ? (int64_t)graph->atom_ids.size() : 0; }

int mdsoap_graph_copy(const mdsoap_graph* graph, int64_t* offsets, int32_t* atoms, int32_t* shifts,
                      double* displacements, double* distance2) {
    if (!graph) return fail(MDSOAP_INVALID_ARGUMENT, "null graph");
    if (offsets) std::memcpy(offsets, graph->offsets.data(), 8 * graph->offsets.size());
    if (atoms && !graph->atom_ids.empty()) std::memcpy(atoms, graph->atom_ids.data(), 4 * graph->atom_ids.size());
    if (shifts && !graph->shifts.empty()) std::memcpy(shifts, graph->shifts.data(), 4 * graph->shifts.size());
    if (displacements && !graph->displacements.empty())
        std::memcpy(displacements, graph->displacements.data(), 8 * graph->displacements.size());
    if (distance2 && !graph->distance2.empty())
        std::memcpy(distance2, graph->distance2.data(), 8 * graph->distance2.size());
    return MDSOAP_OK;
}

void mdsoap_graph_destroy(mdsoap_graph* graph) { delete graph; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Local spherical spectra (SphericalExpansion, SoapRadialSpectrum,
// SoapPowerSpectrum): host tables and driver.

namespace {

struct LocalHostTables {
    int n = 0, lc = 0;
    double c = 0, gf = 0, log_gf = 0;
    std::vector<double> g, log_cg, gratio, ppow, ortho;
};

struct LocalStaging {
    std::mutex mutex;
    PinnedBytes stage[2];
};

LocalStaging& local_staging(int device) {
    // Never destroyed: freeing pinned memory after the CUDA runtime has shut
    // down at process exit is not allowed.
    static std::mutex registry_mutex;
    static auto* registry = new std::map<int, std::unique_ptr<LocalStaging>>();
    std::lock_guard<std::mutex> lock(registry_mutex);
    auto& slot = (*registry)[device];
    if (!slot) slot = std::make_unique<LocalStaging>();
    return *slot;
}

double checked_gamma(double x) {
    const double v = std::tgamma(x);
    if (!std::isfinite(v) || v <= 0.0) raise(MDSOAP_INVALID_ARGUMENT, "local descriptor radial basis is numerically singular");
    return v;
}

// S^(-1/2) of the symmetric overlap matrix by the classical Jacobi method:
// each step zeroes the largest off-diagonal entry (rotation angle
// 0.5 atan2(2 a_pq, a_qq - a_pp)), until it is below 1e-15 or after 100 n^2
// steps; result = V diag(lambda)^(-1/2) V^T.  The pivot order, the angle
// formula and the stopping rule are those of the reference's
// inverse_symmetric_sqrt (cpp/src/common/rotational_math.hpp:15-72): the
// orthonormalisation carries the solver's rounding amplified by the overlap's
// condition number, and the same sequence of rotations reproduces the
// reference's radial basis to the last bit.
std::vector<double> inverse_sqrt_spd(std::vector<double> a, int n) {
    std::vector<double> v((size_t)n * n, 0.0);
    for (int i = 0; i < n; ++i) v[(size_t)i * n + i] = 1.0;
    for (int step = 0; step < 100 * n * n; ++step) {
        int p = 0, q = n > 1 ? 1 : 0;
        double largest = 0.0;
        for (int i = 0; i < n; ++i)
            for (int j = i + 1; j < n; ++j)
                if (std::abs(a[(size_t)i * n + j]) > largest) {
                    largest = std::abs(a[(size_t)i * n + j]);
                    p = i;
                    q = j;
                }
        if (largest < 1e-15) break;
        const double angle = 0.5 * std::atan2(2.0 * a[(size_t)p * n + q], a[(size_t)q * n + q] - a[(size_t)p * n + p]);
        const double c = std::cos(angle), s = std::sin(angle);
        for (int k = 0; k < n; ++k) {
            const double akp = a[(size_t)k * n + p], akq = a[(size_t)k * n + q];
            a[(size_t)k * n + p] = c * akp - s * akq;
            a[(size_t)k * n + q] = s * akp + c * akq;
        }
        for (int k = 0; k < n; ++k) {
            const double apk = a[(size_t)p * n + k], aqk = a[(size_t)q * n + k];
            a[(size_t)p * n + k] = c * apk - s * aqk;
            a[(size_t)q * n + k] = s * apk + c * aqk;
        }
        for (int k = 0; k < n; ++k) {
            const double vkp = v[(size_t)k * n + p], vkq = v[(size_t)k * n + q];
            v[(size_t)k * n + p] = c * vkp - s * vkq;
            v[(size_t)k * n + q] = s * vkp + c * vkq;
        }
    }
    std::vector<double> r((size_t)n * n, 0.0);
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < n; ++j)
            for (int k = 0; k < n; ++k)
                r[(size_t)i * n + j] += v[(size_t)i * n + k] * v[(size_t)j * n + k] / std::sqrt(a[(size_t)k * n + k]);
    for (double x : r)
        if (!std::isfinite(x)) raise(MDSOAP_INVALID_ARGUMENT, "radial overlap matrix is singular, lower max_radial");
    return r;
}

// GTO radial basis of the local spectra (GtoRadialBasis, local_spherical_common.hpp:181-253):
// widths sigma_n = r_c max(sqrt n, 1) / n_radial, overlap of the normalised
// r^n exp(-r^2 / 2 sigma_n^2) functions, orthonormalisation N_n S^(-1/2);
// density factors of prepare_density (:240-253).
LocalHostTables local_tables(const mdsoap_local_params& p, int lc) {
    LocalHostTables t;
    const int n = p.max_radial + 1;
    t.n = n;
    t.lc = lc;
    const double radius = p.cutoff;
    std::vector<double> width(n), norm(n);
    t.g.resize(n);
    for (int k = 0; k < n; ++k) {
        width[k] = radius * std::max(std::sqrt((double)k), 1.0) / n;
        t.g[k] = 1.0 / (2.0 * width[k] * width[k]);
        norm[k] = std::sqrt(2.0 / (std::pow(width[k], 2 * k + 3) * checked_gamma(k + 1.5)));
    }
    std::vector<double> overlap((size_t)n * n);
    for (int a = 0; a < n; ++a)
        for (int b = a; b < n; ++b) {
            const double s1 = width[a], s2 = width[b];
            const double e = 0.5 * (3.0 + a + b);
            const double value = std::pow(0.5 / (s1 * s1) + 0.5 / (s2 * s2), -e) / (std::pow(s1, a) * std::pow(s2, b)) *
                                 checked_gamma(e) /
                                 (std::pow(s1 * s2, 1.5) * std::sqrt(checked_gamma(a + 1.5) * checked_gamma(b + 1.5)));
            overlap[(size_t)a * n + b] = overlap[(size_t)b * n + a] = value;
        }
    const std::vector<double> inv = inverse_sqrt_spd(overlap, n);
    t.ortho.resize((size_t)n * n);
    for (int a = 0; a < n; ++a)
        for (int b = 0; b < n; ++b) t.ortho[(size_t)a * n + b] = norm[a] * inv[(size_t)a * n + b];
    const double w2 = p.density_width * p.density_width;
    t.c = 1.0 / (2.0 * w2);
    t.gf = std::pow(3.141592653589793238462643383279502884 / w2, 0.75);
    t.log_gf = std::log(t.gf);
    t.log_cg.resize(n);
    for (int k = 0; k < n; ++k) t.log_cg[k] = std::log(t.c + t.g[k]);
    t.gratio.resize((size_t)(lc + 1) * n);
    t.ppow.resize((size_t)(lc + 1) * n);
    for (int l = 0; l <= lc; ++l) {
        const double gb = checked_gamma(l + 1.5);
        for (int k = 0; k < n; ++k) {
            const double a = 0.5 * (k + l + 3.0);
            t.gratio[(size_t)l * n + k] = checked_gamma(a) / gb;
            t.ppow[(size_t)l * n + k] = std::pow(t.c + t.g[k], -a);
        }
    }
    return t;
}

void validate_local(const mdsoap_local_params* p) {
    if (!p) raise(MDSOAP_INVALID_ARGUMENT, "null argument");
    // local_common.hpp:12-21 (validate_options)
    if (!std::isfinite(p->cutoff) || p->cutoff <= 0.0 || !std::isfinite(p->density_width) || p->density_width <= 0.0 ||
        p->max_radial < 0 || p->max_angular < 0)
        raise(MDSOAP_INVALID_ARGUMENT, "invalid local descriptor descriptor parameters");
    if (p->kind != MDSOAP_LOCAL_SPHERICAL_EXPANSION && p->kind != MDSOAP_LOCAL_RADIAL_SPECTRUM &&
        p->kind != MDSOAP_LOCAL_POWER_SPECTRUM)
        raise(MDSOAP_INVALID_ARGUMENT, "unknown local descriptor kind");
    if (p->n_species <= 0 || !p->species) raise(MDSOAP_INVALID_ARGUMENT, "species must not be empty");
    for (int i = 0; i < p->n_species; ++i) {
        if (p->species[i] <= 0) raise(MDSOAP_INVALID_ARGUMENT, "species must be positive atomic numbers");
        for (int j = 0; j < i; ++j)
            if (p->species[j] == p->species[i]) raise(MDSOAP_INVALID_ARGUMENT, "species must be unique");
    }
    if (p->max_radial + 1 > kLocalMaxN)
        raise(MDSOAP_INVALID_ARGUMENT, "max_radial above the GPU local spectra limit (15)");
    if (p->max_angular > kLocalMaxL && p->kind != MDSOAP_LOCAL_RADIAL_SPECTRUM)
        raise(MDSOAP_INVALID_ARGUMENT, "max_angular above the GPU local spectra limit (8)");
}

int64_t local_features(const mdsoap_local_params& p) {
    const int64_t S = p.n_species, n = p.max_radial + 1, A = p.max_angular + 1;
    if (p.kind == MDSOAP_LOCAL_RADIAL_SPECTRUM) return S * S * n;
    if (p.kind == MDSOAP_LOCAL_POWER_SPECTRUM) return S * (S + 1) / 2 * S * A * n * n;
    return S * S * n * A * A;
}

}  // namespace

extern "C" {

int64_t mdsoap_local_feature_count(const mdsoap_local_params* params) {
    try {
        validate_local(params);
        return local_features(*params);
    } catch (const Failure& f) {
        fail(f.status, f.message);
        return -1;
    }
}

int mdsoap_local_compute(const mdsoap_local_params* params, const mdsoap_batch* batch, double* out, int32_t device) {
    if (!params || !batch) return fail(MDSOAP_INVALID_ARGUMENT, "null argument");
    try {
        validate_local(params);
        validate_host_batch(nullptr, *batch);
        const int64_t atoms = batch->atoms, S = batch->structures;
        const int64_t features = local_features(*params);
        for (int64_t a = 0; a < atoms; ++a) {
            bool known = false;
            for (int i = 0; i < params->n_species; ++i) known = known || params->species[i] == batch->numbers[a];
            if (!known) raise(MDSOAP_INVALID_ARGUMENT, "batch contains an atomic number outside calculator species");
        }
        if (atoms == 0 || S == 0) return MDSOAP_OK;
        if (!out) raise(MDSOAP_INVALID_ARGUMENT, "null output");
        if (features > 2147483647LL) raise(MDSOAP_INVALID_ARGUMENT, "local descriptor feature count exceeds int32");
        const int lc = params->kind == MDSOAP_LOCAL_RADIAL_SPECTRUM ? 0 : params->max_angular;
        const LocalLayout lay = local_layout(params->n_species, params->max_radial + 1, lc);
        int warps = 4;
        while (warps > 1 && lay.bytes_per_warp * warps > 200 * 1024) --warps;
        if (lay.bytes_per_warp * warps > 227 * 1024)
            raise(MDSOAP_INVALID_ARGUMENT, "local descriptor shape needs more shared memory than a GPU block holds");
        const LocalHostTables ht = local_tables(*params, lc);

        int count = 0;
        const cudaError_t probe_err = cudaGetDeviceCount(&count);
        if (probe_err != cudaSuccess || count == 0)
            raise(MDSOAP_DEVICE_UNAVAILABLE, std::string("no CUDA device available: ") + cudaGetErrorString(probe_err));
        if (device < 0 || device >= count) raise(MDSOAP_DEVICE_UNAVAILABLE, "CUDA device index out of range");
        check(cudaSetDevice(device), "cudaSetDevice");
        cudaStream_t stream = nullptr;
        check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
        struct StreamGuard {
            cudaStream_t s;
            ~StreamGuard() { cudaStreamDestroy(s); }
        } guard{stream};
        Workspace w;
        struct WorkGuard {
            Workspace& w;
            ~WorkGuard() { w.release(); }
        } wguard{w};
        DeviceBytes error, species, tables, rows;
        struct BytesGuard {
            std::vector<DeviceBytes*> list;
            ~BytesGuard() {
                for (auto* b : list) b->release();
            }
        } bguard{{&error, &species, &tables, &rows}};
        w.numbers.reserve(4 * atoms, "numbers");
        w.positions.reserve(24 * atoms, "positions");
        w.cells.reserve(72 * S, "cells");
        w.pbc.reserve(12 * S, "pbc");
        w.offsets.reserve(8 * (S + 1), "offsets");
        check(cudaMemcpyAsync(w.numbers.ptr, batch->numbers, 4 * atoms, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.positions.ptr, batch->positions, 24 * atoms, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.cells.ptr, batch->cells, 72 * S, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.pbc.ptr, batch->pbc, 12 * S, cudaMemcpyHostToDevice, stream), "H2D");
        check(cudaMemcpyAsync(w.offsets.ptr, batch->offsets, 8 * (S + 1), cudaMemcpyHostToDevice, stream), "H2D");
        species.reserve(4 * params->n_species, "species");
        check(cudaMemcpyAsync(species.ptr, params->species, 4 * params->n_species, cudaMemcpyHostToDevice, stream),
              "H2D");
        const int n = ht.n;
        std::vector<double> packed;
        for (const auto* part : {&ht.g, &ht.log_cg, &ht.gratio, &ht.ppow, &ht.ortho})
            packed.insert(packed.end(), part->begin(), part->end());
        // Reciprocals of the 1F1 series denominators (l + 1.5 + k - 1) k, exact
        // products, correctly rounded by the host division.
        const size_t recip_at = packed.size();
        for (int l = 0; l <= lc; ++l)
            for (int k = 0; k < kLocalRecip; ++k)
                packed.push_back(k == 0 ? 0.0 : 1.0 / (((double)l + 1.5 + (double)k - 1.0) * (double)k));
        // Harmonic normalisation sqrt((2l+1)/(4 pi) (l-m)!/(l+m)!), times sqrt 2
        // for m > 0, with the reference's sign (-1)^m.
        const size_t ynorm_at = packed.size();
        for (int l = 0; l <= lc; ++l)
            for (int m = 0; m <= l; ++m) {
                const double pi = 3.141592653589793238462643383279502884;
                double v = std::sqrt((2.0 * l + 1.0) / (4.0 * pi) *
                                     std::exp(std::lgamma(l - m + 1.0) - std::lgamma(l + m + 1.0)));
                if (m > 0) v *= 1.414213562373095048801688724209698079;
                packed.push_back(m % 2 ? -v : v);
            }
        tables.reserve(8 * packed.size(), "local tables");
        check(cudaMemcpyAsync(tables.ptr, packed.data(), 8 * packed.size(), cudaMemcpyHostToDevice, stream), "H2D");
        error.reserve(64, "error");
        check(cudaMemsetAsync(error.ptr, 0, 64, stream), "memset");
        w.reserve_bins(atoms, S);
        DeviceBatch db{w.numbers.as<int32_t>(), w.positions.as<double>(), w.cells.as<double>(), w.pbc.as<int32_t>(),
                       w.offsets.as<int64_t>(), S, atoms};
        bin_structures_kernel<<<(unsigned)S, 256, 0, stream>>>(db, w.bins(error.as<unsigned>()), params->cutoff,
                                                               species.as<int32_t>(), params->n_species);
        check(cudaGetLastError(), "bin kernel");
        LocalTables t;
        t.kind = params->kind;
        t.n = n;
        t.lc = lc;
        t.l_out = params->max_angular;
        t.species = params->n_species;
        t.features = (int)features;
        t.cutoff = params->cutoff;
        t.cutoff2 = params->cutoff * params->cutoff;
        t.c = ht.c;
        t.gf = ht.gf;
        t.log_gf = ht.log_gf;
        const double* tb = tables.as<double>();
        t.g = tb;
        t.log_cg = tb + n;
        t.gratio = tb + 2 * n;
        t.ppow = t.gratio + (size_t)(lc + 1) * n;
        t.ortho = t.ppow + (size_t)(lc + 1) * n;
        t.recip = tb + recip_at;
        t.ynorm = tb + ynorm_at;
        // Rows in blocks of centres (about MDSOAP_BLOCK_BYTES of rows each),
        // double buffered: block i's kernel runs while the host copies block
        // i-1 out of its pinned staging buffer into the caller's rows.  A
        // pinned `out` receives the D2H directly.
        const size_t row_bytes = 8 * (size_t)features;
        const int64_t chunk = std::max<int64_t>(
            warps, std::min<int64_t>(atoms, (int64_t)((size_t)block_bytes_target() / row_bytes)));
        const size_t block_bytes = row_bytes * (size_t)std::min<int64_t>(chunk, atoms);
        const bool direct = is_pinned(out);
        DeviceBytes rows2;
        struct RowsGuard {
            DeviceBytes& r;
            ~RowsGuard() { r.release(); }
        } rguard{rows2};
        // Pinned staging is allocated once per device and kept until exit
        // (pinning host pages costs more than the copy it speeds up); calls on
        // one device take turns on it.
        LocalStaging& staging = local_staging(device);
        std::lock_guard<std::mutex> staging_lock(staging.mutex);
        // Destroyed before staging_lock: on any exit (an exception included)
        // the stream drains first, so no D2H queued below still writes into
        // the staging buffers once another call on this device takes them.
        struct DrainGuard {
            cudaStream_t s;
            ~DrainGuard() { cudaStreamSynchronize(s); }
        } drain_guard{stream};
        PinnedBytes* stage = staging.stage;
        DeviceBytes* rowbuf[2] = {&rows, &rows2};
        rows.reserve(block_bytes, "local rows");
        if (atoms > chunk) rows2.reserve(block_bytes, "local rows");
        if (!direct) {
            stage[0].reserve(block_bytes);
            if (atoms > chunk) stage[1].reserve(block_bytes);
        }
        cudaEvent_t done[2] = {nullptr, nullptr};
        struct EventGuard {
            cudaEvent_t* e;
            ~EventGuard() {
                for (int i = 0; i < 2; ++i)
                    if (e[i]) cudaEventDestroy(e[i]);
            }
        } eguard{done};
        for (int i = 0; i < 2; ++i) check(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming), "event");
        const size_t smem = lay.bytes_per_warp * warps;
        check(cudaFuncSetAttribute(local_spectra_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
              "smem attribute");
        auto drain = [&](int slot, int64_t b0, int64_t b1) {
            check(cudaEventSynchronize(done[slot]), "sync");
            if (!direct)
                parallel_copy(reinterpret_cast<char*>(out + b0 * features), static_cast<const char*>(stage[slot].ptr),
                              row_bytes * (size_t)(b1 - b0));
        };
        int64_t prev0 = -1, prev1 = -1;
        int slot = 0;
        for (int64_t a0 = 0; a0 < atoms; a0 += chunk, slot ^= 1) {
            const int64_t a1 = std::min<int64_t>(atoms, a0 + chunk);
            const unsigned grid = (unsigned)((a1 - a0 + warps - 1) / warps);
            local_spectra_kernel<<<grid, 32 * warps, smem, stream>>>(t, db.positions, w.bins(error.as<unsigned>()),
                                                                     a0, a1, rowbuf[slot]->as<double>());
            check(cudaGetLastError(), "local spectra kernel");
            void* dst = direct ? static_cast<void*>(out + a0 * features) : stage[slot].ptr;
            check(cudaMemcpyAsync(dst, rowbuf[slot]->ptr, row_bytes * (size_t)(a1 - a0), cudaMemcpyDeviceToHost,
                                  stream),
                  "D2H rows");
            check(cudaEventRecord(done[slot], stream), "event record");
            if (prev0 >= 0) drain(slot ^ 1, prev0, prev1);
            prev0 = a0;
            prev1 = a1;
        }
        if (prev0 >= 0) drain(slot ^ 1, prev0, prev1);
        check(cudaStreamSynchronize(stream), "sync");
        unsigned bits = 0;
        check(cudaMemcpy(&bits, error.ptr, sizeof(unsigned), cudaMemcpyDeviceToHost), "error word");
        if (bits)
            raise(bits & (kErrMixedPbc | kErrSingularCell | kErrUnknownSpecies | kErrLocalSeries) ? MDSOAP_INVALID_ARGUMENT
                                                                                                 : MDSOAP_INTERNAL,
                  device_error_text(bits));
        return MDSOAP_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.message);
    } catch (const std::exception& e) {
        return fail(MDSOAP_INTERNAL, e.what());
    }
}

}  // extern "C"
