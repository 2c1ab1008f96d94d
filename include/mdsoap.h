/*
 * mdsoap -- B200 (sm_100a) SOAP engine behind a plain C ABI.
 *
 * The engine computes MDescriptor's GTO SOAP power spectrum (compression
 * "off", average off / inner / outer, optional per-species weights) on the
 * GPU: cell-binned periodic/isolated neighbour search, per-centre spherical
 * expansion c_{nlm}, power spectrum p_{nn'l}.  No torch types, no C++ in the
 * signatures: plain pointers and sizes.  All arithmetic is IEEE fp64; the
 * result is rounded once, to fp32 or fp64, when it is stored.
 *
 * Every function returns an mdsoap_status; on failure mdsoap_last_error()
 * gives a message for the calling thread.
 */
#ifndef MDSOAP_H
#define MDSOAP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MDSOAP_ABI_VERSION 3

/* Status codes.  They mirror the reference plugin's error classes
 * (cpp/cuda/include/mdescriptor/cuda/error.hpp:15-28 and
 * src/mdescriptor/core/errors.py:83-113): INVALID_ARGUMENT -> ValueError,
 * DEVICE_UNAVAILABLE -> CudaUnavailable (ImportError), OUT_OF_MEMORY ->
 * CudaOutOfMemory (MemoryError), CANCELLED -> CudaCancelledError. */
typedef enum {
    MDSOAP_OK = 0,
    MDSOAP_INVALID_ARGUMENT = 1,
    MDSOAP_DEVICE_UNAVAILABLE = 2,
    MDSOAP_OUT_OF_MEMORY = 3,
    MDSOAP_CANCELLED = 4,
    MDSOAP_CAPACITY_OVERFLOW = 5,
    MDSOAP_INTERNAL = 6
} mdsoap_status;

typedef enum { MDSOAP_FLOAT32 = 0, MDSOAP_FLOAT64 = 1 } mdsoap_dtype;

typedef enum { MDSOAP_AVERAGE_OFF = 0, MDSOAP_AVERAGE_INNER = 1, MDSOAP_AVERAGE_OUTER = 2 } mdsoap_average;

/* Power-spectrum layouts (SoapOptions::compression; soap.cpp:373-387, 933-1012). */
typedef enum {
    MDSOAP_COMPRESSION_OFF = 0,       /* all species pairs t1 <= t2, (S n)(S n + 1)/2 (L + 1) features */
    MDSOAP_COMPRESSION_MU2 = 1,       /* one pooled density, n (n + 1)/2 (L + 1) features */
    MDSOAP_COMPRESSION_MU1NU1 = 2,    /* species x pooled density, S n^2 (L + 1) features */
    MDSOAP_COMPRESSION_CROSSOVER = 3  /* same-species pairs only, S n (n + 1)/2 (L + 1) features */
} mdsoap_compression;

/* Radial weighting functions of the neighbour density (soap_weight,
 * soap.cpp:389-420). */
typedef enum {
    MDSOAP_WEIGHTING_NONE = 0,
    MDSOAP_WEIGHTING_POLY = 1,  /* c (1 + 2 x^3 - 3 x^2)^m for r <= r0, else 0; x = r / r0 */
    MDSOAP_WEIGHTING_POW = 2,   /* c / (d + x^m) */
    MDSOAP_WEIGHTING_EXP = 3    /* c / (d + exp(-x)) */
} mdsoap_weighting;

/* SoapOptions::radial_basis (src/mdescriptor/descriptors/_kernels/core.py:79-95). */
typedef enum { MDSOAP_RADIAL_GTO = 0, MDSOAP_RADIAL_POLYNOMIAL = 1 } mdsoap_radial_basis;

/* Descriptor parameters; the fields of the reference's SoapOptions for the
 * GTO basis (cpp/include/mdescriptor/descriptor.hpp:17-43, filled by
 * SoapKernel._ensure_native, _kernels/core.py:207-269). */
typedef struct {
    int32_t n_species;
    const int32_t* species;        /* atomic numbers in declared order (feature order follows it) */
    const double* species_weights; /* n_species entries, or NULL for 1.0 each */
    double r_cut;                  /* > 1 for the GTO basis */
    double sigma;                  /* Gaussian width; graph cutoff = r_cut + sigma*sqrt(-2 ln 1e-3) */
    int32_t n_max;                 /* 1..32 */
    int32_t l_max;                 /* 0..20 */
    const double* alphas;          /* (l_max+1)*n_max, index l*n_max + k */
    const double* betas;           /* (l_max+1)*n_max*n_max, index (l*n_max + n)*n_max + k */
    int32_t average;               /* mdsoap_average */
    int32_t output_dtype;          /* mdsoap_dtype */
    int32_t compression;           /* mdsoap_compression */
    int32_t weighting_function;    /* mdsoap_weighting */
    int32_t weighting_has_w0;      /* non-zero: the exact self pair weighs weighting_w0 */
    double weighting_r0;           /* > 0 when a function is set */
    double weighting_c;            /* >= 0 */
    double weighting_d;            /* >= 0 */
    double weighting_m;            /* >= 0 */
    double weighting_w0;           /* >= 0 */
    /* Radial basis (SoapOptions::radial_basis): 0 GTO (alphas / betas above),
     * 1 polynomial on a quadrature grid (_basis_polynomial,
     * src/mdescriptor/descriptors/_kernels/core.py:79-95): radial_grid and
     * radial_weights [radial_grid_size] (nodes in [0, r_cut], positive
     * weights), radial_values [n_max * radial_grid_size] (the orthonormal
     * basis on the nodes, index n * grid_size + q). */
    int32_t radial_basis;
    int32_t radial_grid_size;      /* 2..128 */
    const double* radial_grid;
    const double* radial_weights;
    const double* radial_values;
} mdsoap_params;

/* A flat batch with StructureBatch's layout (src/mdescriptor/core/input.py:20-131):
 * numbers int32[atoms], positions float64[atoms*3], cells float64[structures*9]
 * (lattice vectors as rows), pbc int32[structures*3] (all 0 or all 1 per
 * structure), offsets int64[structures+1]. */
typedef struct {
    const int32_t* numbers;
    const double* positions;
    const double* cells;
    const int32_t* pbc;
    const int64_t* offsets;
    int64_t structures;
    int64_t atoms;
} mdsoap_batch;

typedef struct mdsoap_plan mdsoap_plan;
typedef struct mdsoap_graph mdsoap_graph;
typedef struct mdsoap_pairs mdsoap_pairs;

/* Cooperative cancellation probe; non-zero means "stop".  Polled between
 * blocks of work, never inside a kernel. */
typedef int (*mdsoap_cancel_fn)(void* context);

/* Thread-local message of the last failing call ("" if none). */
const char* mdsoap_last_error(void);

int32_t mdsoap_abi_version(void);

/* Number of CUDA devices visible to this process (0 when there is no usable
 * driver/device; never fails). */
int32_t mdsoap_device_count(void);

/* Build a plan: validates the parameters and precomputes the radial and
 * harmonic tables.  Touches no GPU (device state is created lazily, per
 * device, on the first compute there).
 * Replaces: the SOAP option parsing and constant upload of
 * compute_soap_descriptor (cpp/cuda/src/extended_descriptors_soap.cuh:806-906)
 * behind Backend::Backend (cpp/cuda/src/backend.cu:296-332); CPU counterpart
 * SoapCalculator::SoapCalculator / prepare_soap (cpp/src/standalone/soap.cpp:1248, 507-572). */
int mdsoap_plan_create(const mdsoap_params* params, mdsoap_plan** plan);

/* Release the plan and every device buffer it holds (idempotent on NULL).
 * Replaces: Backend::close (cpp/cuda/src/backend.cu:720-744). */
void mdsoap_plan_destroy(mdsoap_plan* plan);

/* Features per output row: (S n)(S n + 1)/2 (L + 1)
 * (SoapKernel.feature_count, src/mdescriptor/descriptors/_kernels/core.py:272-284). */
int64_t mdsoap_plan_feature_count(const mdsoap_plan* plan);

/* Output rows for a batch: atoms (average off) or structures (inner/outer). */
int64_t mdsoap_plan_rows(const mdsoap_plan* plan, const mdsoap_batch* batch);

/* End-to-end compute from HOST memory into HOST memory: validates the batch
 * on the host, uploads it, runs the GPU pipeline and copies the rows into
 * `out` (rows * feature_count elements of params.output_dtype, C order).
 * The batch is split into structure blocks that are computed and copied back
 * with the copies overlapping the next block's kernels.  `devices` lists the
 * CUDA devices to shard structures across (NULL / 0 means device 0); each
 * device fills a disjoint row range of `out`.  `cancel` (may be NULL) is
 * polled between blocks.
 * Replaces: Backend::compute -> compute_extended_descriptor ->
 * compute_soap_descriptor (cpp/cuda/src/backend.cu:338-356,570-588;
 * cpp/cuda/src/extended_descriptors_soap.cuh:799-1125) and the upload /
 * download path (cpp/cuda/src/batch.cu, context.cu:111-138). */
int mdsoap_compute(mdsoap_plan* plan, const mdsoap_batch* batch, void* out,
                   const int32_t* devices, int32_t n_devices, mdsoap_cancel_fn cancel,
                   void* cancel_context);

/* Device-resident compute on one device: every pointer of `batch` and `out`
 * is device memory on `device`; work is enqueued on `stream` (a cudaStream_t,
 * NULL for the legacy default stream) and the call returns without waiting.
 * Errors detected on the device (unknown species, int32 image overflow) are
 * reported by mdsoap_plan_check(), which synchronises the stream.
 * Replaces: the device part of compute_soap_descriptor
 * (extended_descriptors_soap.cuh:888-1114: build_dpa, expansion, power). */
int mdsoap_compute_device(mdsoap_plan* plan, const mdsoap_batch* batch, void* out, int32_t device,
                          void* stream);

/* Wait for `stream` and report any error flagged by kernels of this plan on
 * `device` since the last check (and clear it). */
int mdsoap_plan_check(mdsoap_plan* plan, int32_t device, void* stream);

/* Sparse rows.  The feature matrix in CSR form with exact zeros dropped,
 * built on `device`: the batch (host arrays) is uploaded, the rows are
 * computed into device memory, and a count pass, a prefix and a fill pass
 * emit row offsets, column indices and values (columns ascending within a
 * row), so only the nonzeros cross PCIe.  Values have the plan's output dtype;
 * the result equals scipy.sparse.csr_matrix of the dense rows mdsoap_compute
 * returns.  Device memory for the dense rows is allocated for the call and
 * freed before it returns.
 * Replaces: format_values(..., sparse=True) on the dense host matrix
 * (src/mdescriptor/core/result.py:64-84) for OutputOptions(sparse=True). */
typedef struct mdsoap_csr mdsoap_csr;
int mdsoap_compute_csr(mdsoap_plan* plan, const mdsoap_batch* batch, int32_t device, mdsoap_csr** csr);
/* Shape and number of stored values of a CSR result. */
int mdsoap_csr_info(const mdsoap_csr* csr, int64_t* rows, int64_t* cols, int64_t* nnz);
/* Copy out: indptr int64[rows + 1], indices int32[nnz], data [nnz] of the
 * plan's output dtype. */
int mdsoap_csr_copy(const mdsoap_csr* csr, int64_t* indptr, int32_t* indices, void* data);
void mdsoap_csr_destroy(mdsoap_csr* csr);

/* Size of the fixed device scratch area used by mdsoap_compute_device_noalloc:
 * 32 MiB, held by every GPU that loads this library until the process exits. */
#define MDSOAP_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)

/* Device-resident compute that allocates no memory (this entry point has no
 * counterpart in the reference).
 *
 * For callers that cannot allocate device memory while they run: a process
 * whose framework allocator has already reserved the GPU's memory (a cudaMalloc
 * would fail or fragment that pool), or a latency-critical loop that must not
 * take the device-wide synchronisation cudaMalloc/cudaFree imply.  Such a
 * caller passes device inputs and a device output exactly as for
 * mdsoap_compute_device; every working buffer (neighbour bins, copies of the
 * plan's radial tables, the error word, per-centre coefficient blocks for the
 * averages) lives in one file-scope __device__ array of
 * MDSOAP_NOALLOC_SCRATCH_BYTES, and the call makes no cudaMalloc, cudaFree or
 * other allocating call.
 *
 * Limits and rules:
 *  - A batch whose working set does not fit the scratch array is rejected with
 *    MDSOAP_CAPACITY_OVERFLOW before any device work (roughly 76 bytes per atom
 *    plus 300 per structure for average "off"; the averages add one
 *    coefficient block or feature row per atom).
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress, with `device` made current) and raises the
 *    kernels' shared-memory limit; make that first call before any stream
 *    capture.
 *  - All calls in the process share the one array and it keeps the last
 *    call's contents; everything that must start at zero is cleared by each
 *    call.  Calls whose GPU work overlaps (different streams or threads)
 *    race on the array: serialise them.
 *  - Every call blocks: after queueing its kernels it copies the error word
 *    back to the host and calls cudaStreamSynchronize(stream), so it returns
 *    only once its work on `stream` has finished, with device-detected input
 *    errors (unknown species, mixed pbc, singular cell) as its status. */
int mdsoap_compute_device_noalloc(mdsoap_plan* plan, const mdsoap_batch* batch, void* out, int32_t device,
                                  void* stream);

/* Page-locked host buffers for result rows, recycled across calls (no
 * counterpart in the reference; used by the plugin for the rows it returns).
 * Rows written into such a buffer by mdsoap_compute leave the GPU by a direct
 * D2H, and a recycled buffer's pages are already resident, so neither the
 * staging copy nor first-touch page faults of a fresh pageable array are paid.
 * acquire: a buffer of at least `bytes` from the idle pool (a cached one at
 * most twice as large) or newly page-locked; MDSOAP_OUT_OF_MEMORY when the
 * host refuses to lock more memory.  release: back to the idle pool, which
 * keeps at most MDSOAP_HOST_POOL_BYTES (environment, default 4 GiB; 0
 * disables the pool's caching) and unlocks the rest.  Buffers are never
 * unlocked at process exit.  Thread-safe. */
int mdsoap_host_buffer_acquire(size_t bytes, void** ptr);
void mdsoap_host_buffer_release(void* ptr);

/* Per-kernel CUDA-event timing of mdsoap_compute_device calls (measurement
 * support; no counterpart in the reference).  While enabled, each device call
 * records events around its binning, centre and structure kernels on the
 * caller's stream; mdsoap_plan_last_timing waits for them and returns the
 * milliseconds of the last call on `device`. */
int mdsoap_plan_set_timing(mdsoap_plan* plan, int32_t enable);
int mdsoap_plan_last_timing(mdsoap_plan* plan, int32_t device, double* bin_ms, double* center_ms,
                            double* structure_ms);

/* The centre time of the last timed call split into the expansion kernel and
 * the separate tail kernel (beta transform + power spectrum) that split-tail
 * plans launch after it, each summed over the chunks of centres the call ran
 * as expansion / tail launch pairs; tail_ms is 0 when the plan runs a fused
 * tail (measurement support; no counterpart in the reference). */
int mdsoap_plan_last_timing_split(mdsoap_plan* plan, int32_t device, double* expansion_ms, double* tail_ms);

/* Number of kernels the plan has launched so far, over all devices and entry
 * points (measurement support; no counterpart in the reference).  A
 * benchmark reads it before and after its timed region to count its launches. */
int mdsoap_plan_launch_count(const mdsoap_plan* plan, int64_t* count);

/* Name and template arguments of the centre kernel(s) the plan launches, e.g.
 * "soap_paired_kernel<4, 6, false, 2> + soap_tail_kernel<6, 4>" (measurement
 * support, for matching profiler records; no counterpart in the reference).
 * Never NULL; valid while the plan lives. */
const char* mdsoap_plan_kernel(const mdsoap_plan* plan);

/* The engine's exp() for non-positive arguments (Tang's table-driven
 * method, used for every radial factor exp(-a r^2)) and CUDA's exp(), both
 * evaluated on `device` for `count` host arguments; results are written to
 * the host arrays `ours` and `cuda_exp` (test support; no counterpart in the
 * reference, whose CPU path calls std::exp, soap.cpp:895-896). */
int mdsoap_probe_exp(int32_t device, const double* x, int64_t count, double* ours, double* cuda_exp);

/* The radial factors pref * exp(-e u) as the kernels form them, beside
 * pref * CUDA's exp(-e u), on `device` for `count` host triples (u, e, pref),
 * written to the host arrays `ours` and `cuda_exp`.  form 0: the float64-row
 * form; 1: the float32-row form of the one-kernel walk; 2: the float32-row
 * form of the expansion-only kernel (exponent folded into the reduction,
 * 64-entry table).  The caller keeps e u in [0, 700] and the result a normal
 * double, as the plans do (test support; no counterpart in the reference,
 * whose CPU path calls std::exp, soap.cpp:895-896). */
int mdsoap_probe_radial(int32_t device, int32_t form, const double* u, const double* e, const double* pref,
                        int64_t count, double* ours, double* cuda_exp);

/* Failure-detection probe (test support; no counterpart in the reference):
 * launches one thread that arms an mbarrier for a bulk copy it never issues
 * and waits for it with the tail kernel's own bounded wait (limit_ns, at most
 * 2 s).  The wait runs out, the kernel sets the tail-timeout bit of its error
 * word and returns; the call then reports MDSOAP_INTERNAL ("tail kernel: a
 * coefficient block copy did not complete in time"), as mdsoap_compute does
 * when a real copy stalls.  Nothing is left in flight, so the device stays
 * usable.  MDSOAP_OK would mean the wait did not run out. */
int mdsoap_probe_bounded_wait(int32_t device, uint64_t limit_ns);

/* Measured fp64 FMA throughput of `device` in TFLOP/s (2 flops per FMA) from a
 * register-resident FMA chain kernel over every SM (measurement support; no
 * counterpart in the reference).  Used as the roofline denominator of the
 * fp64-bound centre kernel. */
int mdsoap_probe_fp64_fma(int32_t device, double* tflops);

/* Neighbour graph of a host batch on `device` with an explicit cutoff:
 * inclusive boundary, exact self pair kept, periodic images as integer
 * shifts of the unwrapped positions.  The pair SET and the fp64
 * displacement / squared-distance bits equal the reference CPU graph's; pairs
 * of one centre come in the engine's (deterministic) cell order.
 * Replaces: DeviceNeighborGraph::build_dpa (cpp/cuda/src/neighbor_graph.cu:1106-1363);
 * CPU counterpart build_neighbor_graph (cpp/src/common/neighbor.cpp:703-768). */
int mdsoap_graph_build(const mdsoap_batch* batch, double cutoff, int32_t device,
                       mdsoap_graph** graph);

int64_t mdsoap_graph_pairs(const mdsoap_graph* graph);

/* Copy the CSR out: offsets int64[atoms+1], atoms int32[pairs] (batch-global
 * indices), shifts int32[pairs*3], displacements float64[pairs*3],
 * distance2 float64[pairs].  Any pointer may be NULL to skip that array. */
int mdsoap_graph_copy(const mdsoap_graph* graph, int64_t* offsets, int32_t* atoms, int32_t* shifts,
                      double* displacements, double* distance2);

void mdsoap_graph_destroy(mdsoap_graph* graph);

/* The NeighborList descriptor of a host batch, computed on `device`: every
 * pair within `cutoff` (inclusive), without the exact self pair unless
 * `self_pairs`, and only one orientation of each pair unless `full_list`
 * (keep_half_neighbor: the larger atom index, ties broken by the first
 * non-zero image shift being positive).  Rows come in the reference's order
 * (centre by centre, then the reference cell-list order within a centre).
 * A centre may hold at most 2048 listed pairs (MDSOAP_CAPACITY_OVERFLOW beyond).
 * Replaces: compute_neighbor_list (cpp/src/standalone/neighbor_list.cpp:15-75)
 * and the reference plugin's NeighborList branch (cpp/cuda/src/backend.cu:358-471). */
int mdsoap_neighbor_list(const mdsoap_batch* batch, double cutoff, int32_t full_list, int32_t self_pairs,
                         int32_t device, mdsoap_pairs** pairs);

int64_t mdsoap_pairs_count(const mdsoap_pairs* pairs);

/* Copy the table out: records float64[pairs*5] = (centre, atom, shift a, shift
 * b, shift c) with batch-global atom indices, values float64[pairs*4] = (dx,
 * dy, dz, distance), row_offsets int64[structures+1] = first row of each
 * structure.  Any pointer may be NULL to skip that array. */
int mdsoap_pairs_copy(const mdsoap_pairs* pairs, double* records, double* values, int64_t* row_offsets);

void mdsoap_pairs_destroy(mdsoap_pairs* pairs);

/* Local spherical spectra: the featomic-style GTO expansion of a Gaussian
 * atomic density (width `density_width`) with a cosine cutoff of width
 * min(0.5, cutoff).  `kind` takes the reference's LocalDescriptorKind values:
 * 0 SphericalExpansion, 2 SoapRadialSpectrum, 3 SoapPowerSpectrum.  Species
 * are kept in declared order (not sorted), as the reference does. */
#define MDSOAP_LOCAL_SPHERICAL_EXPANSION 0
#define MDSOAP_LOCAL_RADIAL_SPECTRUM 2
#define MDSOAP_LOCAL_POWER_SPECTRUM 3

typedef struct mdsoap_local_params {
    int32_t kind;
    int32_t max_radial;  /* radial count = max_radial + 1, at most 16 */
    int32_t max_angular; /* at most 8 (any value for the radial spectrum) */
    int32_t n_species;
    const int32_t* species;
    double cutoff;
    double density_width;
} mdsoap_local_params;

/* Feature count of one row: S*S*n*(L+1)^2 (expansion), S*S*n (radial
 * spectrum), S(S+1)/2*S*(L+1)*n*n (power spectrum); -1 on invalid options
 * (message in mdsoap_last_error).
 * Replaces: local_descriptor_feature_count (cpp/src/standalone/spherical_expansion.cpp:115-121)
 * and local_layout_feature_count (cpp/src/common/local_layout.hpp:115-130). */
int64_t mdsoap_local_feature_count(const mdsoap_local_params* params);

/* Rows float64[atoms][features] of a host batch computed on `device`, written
 * into the caller's host buffer `out` (atoms * features doubles).
 * Replaces: compute_spherical_expansion (cpp/src/standalone/spherical_expansion.cpp:124-206)
 * and compute_local_descriptors_into, the reference plugin's local branch
 * (cpp/cuda/src/backend.cu:590-624). */
int mdsoap_local_compute(const mdsoap_local_params* params, const mdsoap_batch* batch, double* out,
                         int32_t device);

#ifdef __cplusplus
}
#endif

#endif /* MDSOAP_H */
