/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the SOAP hot path.
 *
 * A plain-C restatement of MDescriptor's CPU SOAP path (GTO radial basis,
 * compression off, average off/inner/outer, optional species weights):
 *   - neighbour graph: cpp/src/common/neighbor.cpp:423-679 (build_structure_graph,
 *     store_shifts=true, include_boundary=true, unscaled images), build_grid
 *     :135-194, CellGrid::coordinate :122-132, inverse/bounds math3.hpp:52-68 and
 *     neighbor.cpp:455-468, image order :519-528, query :558-574, serial append
 *     :579-608, batch concatenation :742-767;
 *   - SOAP: cpp/src/standalone/soap.cpp:1149-1246 (compute_soap), prepare_soap
 *     :507-572, solid harmonics :101-216 (the Cartesian recurrence, used here for
 *     every l; the reference's literal l<=4 / l=6 tables and l>6 Legendre form
 *     are the same functions), species-sorted accumulation :737-760 and
 *     :881-929, power spectrum :997-1012, inner/outer averages :1019-1120.
 *
 * Floating-point order follows the reference expressions (no FMA contraction:
 * the build passes -ffp-contract=off), so the neighbour graph is bit-identical
 * to the reference's and the features agree to rounding.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load this library;
 * the product never does.
 *
 * Extended-precision build (-DORACLE_EXTENDED, liboracle_soap_ext.so): the
 * SOAP stage -- harmonics, radial factors, neighbour sums, beta transform,
 * power spectrum, averages -- runs in x87 extended precision (long double,
 * 64-bit significand, unit roundoff 5.4e-20) on the same double inputs: the
 * same double neighbour graph (displacements and squared distances), the
 * same double plan constants (radial prefactors and exponents, harmonic
 * normalisation, beta, power prefactors) and the same statements.  Its rows
 * are the exact value of the reference's algorithm for those inputs up to
 * ~1e-16 relative, 2^11 times closer than any double evaluation: the
 * yardstick the tests use to measure how far double implementations (the
 * reference's, this checker's, the GPU's) each stray from it.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* Arithmetic type of the SOAP stage (see the header comment). */
#ifdef ORACLE_EXTENDED
typedef long double oreal;
#define OEXP expl
#else
typedef double oreal;
#define OEXP exp
#endif

#define OR_PI 3.141592653589793238462643383279502884
#define OR_SQRT2 1.414213562373095048801688724209698079

static _Thread_local char g_error[256];

static int fail(const char* message) {
    strncpy(g_error, message, sizeof(g_error) - 1);
    g_error[sizeof(g_error) - 1] = '\0';
    return 1;
}

const char* oracle_last_error(void) { return g_error; }

/* ---------------------------------------------------------------- graph -- */

typedef struct {
    int64_t count, capacity;
    int32_t* atoms;
    int32_t* shifts;
    double* displacements;
    double* distance2;
} pair_list;

static int pair_push(pair_list* list, int32_t atom, const int32_t shift[3], const double d[3],
                     double distance2) {
    if (list->count == list->capacity) {
        int64_t capacity = list->capacity ? list->capacity * 2 : 1024;
        int32_t* atoms = realloc(list->atoms, (size_t)capacity * sizeof(int32_t));
        if (!atoms) return 1;
        list->atoms = atoms;
        int32_t* shifts = realloc(list->shifts, (size_t)capacity * 3 * sizeof(int32_t));
        if (!shifts) return 1;
        list->shifts = shifts;
        double* displacements = realloc(list->displacements, (size_t)capacity * 3 * sizeof(double));
        if (!displacements) return 1;
        list->displacements = displacements;
        double* d2 = realloc(list->distance2, (size_t)capacity * sizeof(double));
        if (!d2) return 1;
        list->distance2 = d2;
        list->capacity = capacity;
    }
    int64_t i = list->count++;
    list->atoms[i] = atom;
    memcpy(list->shifts + 3 * i, shift, 3 * sizeof(int32_t));
    memcpy(list->displacements + 3 * i, d, 3 * sizeof(double));
    list->distance2[i] = distance2;
    return 0;
}

static void pair_free(pair_list* list) {
    free(list->atoms);
    free(list->shifts);
    free(list->displacements);
    free(list->distance2);
    memset(list, 0, sizeof(*list));
}

typedef struct {
    int32_t atom;
    int32_t shift[3];
    double position[3];
} extended_atom;

/* CellGrid::coordinate, neighbor.cpp:122-132 */
static int grid_coordinate(double value, double origin, double width, int dimension) {
    const double scaled = (value - origin) / width;
    if (!(scaled > 0.0)) return 0;
    if (!isfinite(scaled) || scaled >= (double)dimension) return dimension - 1;
    return (int)scaled;
}

/* math3.hpp:44-68 (determinant, inverse) */
static int inverse3(const double m[9], double r[9]) {
    const double det = m[0] * (m[4] * m[8] - m[5] * m[7]) - m[1] * (m[3] * m[8] - m[5] * m[6])
                       + m[2] * (m[3] * m[7] - m[4] * m[6]);
    if (!isfinite(det) || fabs(det) < 1e-14) return 1;
    r[0] = (m[4] * m[8] - m[5] * m[7]) / det;
    r[1] = (m[2] * m[7] - m[1] * m[8]) / det;
    r[2] = (m[1] * m[5] - m[2] * m[4]) / det;
    r[3] = (m[5] * m[6] - m[3] * m[8]) / det;
    r[4] = (m[0] * m[8] - m[2] * m[6]) / det;
    r[5] = (m[2] * m[3] - m[0] * m[5]) / det;
    r[6] = (m[3] * m[7] - m[4] * m[6]) / det;
    r[7] = (m[1] * m[6] - m[0] * m[7]) / det;
    r[8] = (m[0] * m[4] - m[1] * m[3]) / det;
    return 0;
}

/*
 * One structure's graph (neighbor.cpp:423-679).  `begin`/`end` index the batch;
 * emitted atom indices are `index_base + local` with local in [0, end-begin).
 * counts has end-begin+1 entries, relative to the list's size on entry.
 */
static int structure_graph(const double* positions, const double* cell, const int32_t* pbc,
                           int64_t begin, int64_t end, double cutoff, int64_t index_base,
                           const int64_t* subset, int64_t subset_count, pair_list* out, int64_t* counts) {
    const int periodic = pbc[0] == 1 && pbc[1] == 1 && pbc[2] == 1;
    const int isolated = pbc[0] == 0 && pbc[1] == 0 && pbc[2] == 0;
    if (!periodic && !isolated) return fail("mixed periodicity is not supported; use all-zero or all-one pbc");
    const int64_t atom_count = end - begin;
    int bounds[3] = {0, 0, 0};
    if (periodic) {
        double inv[9];
        if (inverse3(cell, inv)) return fail("cell matrix is singular");
        for (int a = 0; a < 3; ++a) {
            const double b = floor(cutoff * sqrt(inv[0 * 3 + a] * inv[0 * 3 + a] + inv[1 * 3 + a] * inv[1 * 3 + a]
                                                 + inv[2 * 3 + a] * inv[2 * 3 + a]) + 1.0);
            if (!isfinite(b) || b < 0.0 || b > 2147483647.0) return fail("periodic image range exceeds integer range");
            bounds[a] = (int)b;
        }
    }
    const int64_t images = (int64_t)(2 * bounds[0] + 1) * (2 * bounds[1] + 1) * (2 * bounds[2] + 1);
    const int64_t extended_count = images * atom_count;
    extended_atom* extended = malloc((size_t)(extended_count ? extended_count : 1) * sizeof(extended_atom));
    if (!extended) return fail("out of memory");
    int64_t e = 0;
    /* image order n0 -> n1 -> n2, then atoms (neighbor.cpp:519-528, 471-498) */
    for (int n0 = -bounds[0]; n0 <= bounds[0]; ++n0) {
        for (int n1 = -bounds[1]; n1 <= bounds[1]; ++n1) {
            for (int n2 = -bounds[2]; n2 <= bounds[2]; ++n2) {
                double shift[3];
                for (int c = 0; c < 3; ++c) {
                    const double t0 = (double)n0 * cell[0 * 3 + c];
                    const double t1 = (double)n1 * cell[1 * 3 + c];
                    const double t2 = (double)n2 * cell[2 * 3 + c];
                    shift[c] = (t0 + t1) + t2;
                }
                for (int64_t atom = begin; atom < end; ++atom) {
                    extended_atom* x = &extended[e++];
                    x->atom = (int32_t)(index_base + (atom - begin));
                    x->shift[0] = n0;
                    x->shift[1] = n1;
                    x->shift[2] = n2;
                    /* isolated structures keep the original position (neighbor.cpp:499-502) */
                    for (int c = 0; c < 3; ++c)
                        x->position[c] = periodic ? positions[3 * atom + c] + shift[c] : positions[3 * atom + c];
                }
            }
        }
    }
    /* build_grid, neighbor.cpp:135-194 */
    double minimum[3] = {0, 0, 0}, maximum[3] = {0, 0, 0}, spacing[3] = {0, 0, 0};
    int dims[3] = {1, 1, 1};
    int64_t* cell_offsets = NULL;
    int32_t* cell_atoms = NULL;
    if (extended_count > 0) {
        for (int c = 0; c < 3; ++c) minimum[c] = maximum[c] = extended[0].position[c];
        for (int64_t i = 0; i < extended_count; ++i) {
            for (int c = 0; c < 3; ++c) {
                const double v = extended[i].position[c];
                if (v < minimum[c]) minimum[c] = v;
                if (v > maximum[c]) maximum[c] = v;
            }
        }
        for (int c = 0; c < 3; ++c) {
            minimum[c] -= 1e-10;
            maximum[c] += 1e-10;
            const double range = maximum[c] - minimum[c];
            const double cells = range / cutoff;
            if (!isfinite(range) || range < 0.0 || !isfinite(cells) || cells > 2147483647.0) {
                free(extended);
                return fail("neighbor cell-grid dimension exceeds integer range");
            }
            dims[c] = (int)cells > 1 ? (int)cells : 1;
            const double width = range / dims[c];
            spacing[c] = cutoff > width ? cutoff : width;
        }
        const int64_t cell_count = (int64_t)dims[0] * dims[1] * dims[2];
        cell_offsets = calloc((size_t)cell_count + 1, sizeof(int64_t));
        int64_t* fill = calloc((size_t)cell_count, sizeof(int64_t));
        int32_t* cell_of = malloc((size_t)extended_count * sizeof(int32_t));
        cell_atoms = malloc((size_t)extended_count * sizeof(int32_t));
        if (!cell_offsets || !fill || !cell_of || !cell_atoms) {
            free(extended); free(cell_offsets); free(fill); free(cell_of); free(cell_atoms);
            return fail("out of memory");
        }
        for (int64_t i = 0; i < extended_count; ++i) {
            const int x = grid_coordinate(extended[i].position[0], minimum[0], spacing[0], dims[0]);
            const int y = grid_coordinate(extended[i].position[1], minimum[1], spacing[1], dims[1]);
            const int z = grid_coordinate(extended[i].position[2], minimum[2], spacing[2], dims[2]);
            cell_of[i] = (int32_t)(x + (int64_t)dims[0] * (y + (int64_t)dims[1] * z));
            ++cell_offsets[cell_of[i] + 1];
        }
        for (int64_t c = 0; c < cell_count; ++c) cell_offsets[c + 1] += cell_offsets[c];
        for (int64_t i = 0; i < extended_count; ++i) {
            const int32_t c = cell_of[i];
            cell_atoms[cell_offsets[c] + fill[c]++] = (int32_t)i;
        }
        free(fill);
        free(cell_of);
    }
    /* query + serial append, neighbor.cpp:552-608 */
    const double cutoff2 = cutoff * cutoff;
    const int64_t base = out->count;
    const int64_t queries = subset ? subset_count : atom_count;
    for (int64_t q = 0; q < queries; ++q) {
        const int64_t local = subset ? subset[q] : q;
        counts[q] = out->count - base;
        if (extended_count == 0) continue;
        const double* center = positions + 3 * (begin + local);
        const int ix = grid_coordinate(center[0], minimum[0], spacing[0], dims[0]);
        const int iy = grid_coordinate(center[1], minimum[1], spacing[1], dims[1]);
        const int iz = grid_coordinate(center[2], minimum[2], spacing[2], dims[2]);
        for (int z = iz - 1 > 0 ? iz - 1 : 0; z <= (iz + 1 < dims[2] - 1 ? iz + 1 : dims[2] - 1); ++z) {
            for (int y = iy - 1 > 0 ? iy - 1 : 0; y <= (iy + 1 < dims[1] - 1 ? iy + 1 : dims[1] - 1); ++y) {
                for (int x = ix - 1 > 0 ? ix - 1 : 0; x <= (ix + 1 < dims[0] - 1 ? ix + 1 : dims[0] - 1); ++x) {
                    const int64_t c = x + (int64_t)dims[0] * (y + (int64_t)dims[1] * z);
                    for (int64_t o = cell_offsets[c]; o < cell_offsets[c + 1]; ++o) {
                        const extended_atom* n = &extended[cell_atoms[o]];
                        const double d[3] = {n->position[0] - center[0], n->position[1] - center[1],
                                             n->position[2] - center[2]};
                        const double distance2 = d[0] * d[0] + d[1] * d[1] + d[2] * d[2];
                        if (!(distance2 <= cutoff2)) continue;
                        if (pair_push(out, n->atom, n->shift, d, distance2)) {
                            free(extended); free(cell_offsets); free(cell_atoms);
                            return fail("out of memory");
                        }
                    }
                }
            }
        }
    }
    counts[queries] = out->count - base;
    free(extended);
    free(cell_offsets);
    free(cell_atoms);
    return 0;
}

typedef struct {
    int64_t atoms;
    int64_t* offsets;
    pair_list pairs;
} oracle_graph;

static int validate_batch(const int32_t* numbers, const double* positions, const double* cells,
                          const int32_t* pbc, const int64_t* offsets, int64_t structures) {
    if (structures < 0 || !offsets) return fail("invalid structure batch");
    if (offsets[0] != 0) return fail("offsets do not describe the flattened arrays");
    for (int64_t s = 0; s < structures; ++s) {
        if (offsets[s + 1] < offsets[s]) return fail("offsets must be monotonic");
        int periodic = 1, isolated = 1;
        for (int a = 0; a < 3; ++a) {
            if (pbc[3 * s + a] != 0 && pbc[3 * s + a] != 1) return fail("pbc must contain only 0 or 1");
            periodic = periodic && pbc[3 * s + a] == 1;
            isolated = isolated && pbc[3 * s + a] == 0;
        }
        if (!periodic && !isolated) return fail("mixed periodicity is not supported; use all-zero or all-one pbc");
        for (int k = 0; k < 9; ++k)
            if (!isfinite(cells[9 * s + k])) return fail("cells must be finite");
    }
    for (int64_t i = 0; i < offsets[structures]; ++i) {
        if (numbers[i] <= 0) return fail("atomic numbers must be positive");
        for (int a = 0; a < 3; ++a)
            if (!isfinite(positions[3 * i + a])) return fail("positions must be finite");
    }
    return 0;
}

/* build_neighbor_graph over a whole batch (neighbor.cpp:703-768): global atom
 * indices, structures concatenated in order. */
void* oracle_graph_build(const int32_t* numbers, const double* positions, const double* cells,
                         const int32_t* pbc, const int64_t* offsets, int64_t structures,
                         double cutoff) {
    if (!isfinite(cutoff) || cutoff <= 0.0) {
        fail("neighbor cutoff must be finite and positive");
        return NULL;
    }
    if (validate_batch(numbers, positions, cells, pbc, offsets, structures)) return NULL;
    oracle_graph* g = calloc(1, sizeof(oracle_graph));
    const int64_t atoms = offsets[structures];
    g->atoms = atoms;
    g->offsets = calloc((size_t)atoms + 2, sizeof(int64_t));
    int64_t* counts = malloc(((size_t)atoms + 2) * sizeof(int64_t));
    for (int64_t s = 0; s < structures; ++s) {
        const int64_t begin = offsets[s], end = offsets[s + 1];
        const int64_t before = g->pairs.count;
        if (structure_graph(positions, cells + 9 * s, pbc + 3 * s, begin, end, cutoff, begin, NULL, 0,
                            &g->pairs, counts)) {
            free(counts);
            pair_free(&g->pairs);
            free(g->offsets);
            free(g);
            return NULL;
        }
        for (int64_t local = 0; local <= end - begin; ++local) g->offsets[begin + local] = before + counts[local];
    }
    if (structures == 0) g->offsets[0] = 0;
    free(counts);
    return g;
}

int64_t oracle_graph_pairs(void* handle) { return ((oracle_graph*)handle)->pairs.count; }

void oracle_graph_copy(void* handle, int64_t* offsets, int32_t* atoms, int32_t* shifts,
                       double* displacements, double* distance2) {
    oracle_graph* g = handle;
    const int64_t p = g->pairs.count;
    memcpy(offsets, g->offsets, ((size_t)g->atoms + 1) * sizeof(int64_t));
    if (p) {
        memcpy(atoms, g->pairs.atoms, (size_t)p * sizeof(int32_t));
        memcpy(shifts, g->pairs.shifts, (size_t)p * 3 * sizeof(int32_t));
        memcpy(displacements, g->pairs.displacements, (size_t)p * 3 * sizeof(double));
        memcpy(distance2, g->pairs.distance2, (size_t)p * sizeof(double));
    }
}

void oracle_graph_free(void* handle) {
    oracle_graph* g = handle;
    if (!g) return;
    pair_free(&g->pairs);
    free(g->offsets);
    free(g);
}

/* ----------------------------------------------------------------- SOAP -- */

typedef struct {
    int n_species, n_max, l_max, width, harmonics;
    int compression;            /* 0 off, 1 mu2, 2 mu1nu1, 3 crossover */
    int weighting_function;     /* 0 none, 1 poly, 2 pow, 3 exp */
    int weighting_has_w0;
    double weighting_r0, weighting_c, weighting_d, weighting_m, weighting_w0;
    const int32_t* species;
    const double* species_weights;
    const double* betas;
    double soap_scale;
    double* power_prefactors;   /* [L+1] */
    double* normalization;      /* [(L+1)^2], l*width+m */
    double* radial_prefactors;  /* [(L+1)*n] */
    double* radial_exponents;   /* [(L+1)*n] */
    int radial_basis;           /* 0 GTO, 1 polynomial */
    int grid_size;              /* polynomial: quadrature nodes Q */
    const double* grid;         /* [Q] */
    double* weighted_values;    /* [Q][n]: weight_q grid_q^2 values[n][q] (soap.cpp:555-569) */
    double eta;
} soap_plan;

/* Real regular solid harmonics r^l Y_lm, layout l^2 + (l-m) = cos m, l^2 + l = m0,
 * l^2 + (l+m) = sin m (soap.cpp:101-216, generic Cartesian recurrence). */
static void solid_harmonics(const soap_plan* plan, oreal x, oreal y, oreal z, oreal r2,
                            oreal* real, oreal* imag, oreal* result) {
    const int L = plan->l_max, w = plan->width;
    for (int i = 0; i < w * w; ++i) real[i] = imag[i] = 0.0;
    real[0] = 1.0;
    for (int m = 0; m <= L; ++m) {
        if (m > 0) {
            const double factor = -(2.0 * m - 1.0);
            const oreal pr = real[(m - 1) * w + (m - 1)], pi = imag[(m - 1) * w + (m - 1)];
            real[m * w + m] = factor * (x * pr - y * pi);
            imag[m * w + m] = factor * (x * pi + y * pr);
        }
        if (m == 0) {
            if (L >= 1) real[1 * w + 0] = z;
            for (int l = 2; l <= L; ++l)
                real[l * w] = ((2.0 * l - 1.0) * z * real[(l - 1) * w] - (l - 1.0) * r2 * real[(l - 2) * w]) / l;
        } else {
            if (m < L) {
                real[(m + 1) * w + m] = (2.0 * m + 1.0) * z * real[m * w + m];
                imag[(m + 1) * w + m] = (2.0 * m + 1.0) * z * imag[m * w + m];
            }
            for (int l = m + 2; l <= L; ++l) {
                real[l * w + m] = ((2.0 * l - 1.0) * z * real[(l - 1) * w + m]
                                   - (l + m - 1.0) * r2 * real[(l - 2) * w + m]) / (l - m);
                imag[l * w + m] = ((2.0 * l - 1.0) * z * imag[(l - 1) * w + m]
                                   - (l + m - 1.0) * r2 * imag[(l - 2) * w + m]) / (l - m);
            }
        }
    }
    for (int l = 0; l <= L; ++l) {
        result[l * l + l] = plan->normalization[l * w] * real[l * w];
        for (int m = 1; m <= l; ++m) {
            const double factor = OR_SQRT2 * plan->normalization[l * w + m];
            result[l * l + (l - m)] = factor * real[l * w + m];
            result[l * l + (l + m)] = factor * imag[l * w + m];
        }
    }
}

/* soap_weight (soap.cpp:389-420): weighting function of the distance, w0 for
 * the exact self pair, times the species weight. */
static double soap_weight(const soap_plan* plan, double distance, int exact_self, int type) {
    double value = 1.0;
    if (plan->weighting_function != 0) {
        const double ratio = distance / plan->weighting_r0;
        if (plan->weighting_function == 1) {
            value = distance > plan->weighting_r0
                        ? 0.0
                        : plan->weighting_c * pow(1.0 + 2.0 * ratio * ratio * ratio - 3.0 * ratio * ratio,
                                                  plan->weighting_m);
        } else if (plan->weighting_function == 2) {
            value = plan->weighting_c / (plan->weighting_d + pow(ratio, plan->weighting_m));
        } else {
            value = plan->weighting_c / (plan->weighting_d + exp(-ratio));
        }
    }
    if (exact_self && plan->weighting_has_w0) value = plan->weighting_w0;
    return value * plan->species_weights[type];
}

static int species_type(const soap_plan* plan, int32_t z) {
    for (int t = 0; t < plan->n_species; ++t)
        if (plan->species[t] == z) return t;
    return -1;
}

/* Conditioning probe for tests: when set, every exponential of the polynomial
 * basis is moved by one unit in the last place (up or down by a bit of its
 * argument), so a test can measure how far last-bit differences between exp
 * implementations travel through the reference's flir recurrence. */
static int g_flir_exp_ulp = 0;

void oracle_set_flir_exp_ulp(int enabled) { g_flir_exp_ulp = enabled; }

static double flir_exp(double x) {
    double v = exp(x);
    if (g_flir_exp_ulp && v > 0.0) {
        uint64_t a, b;
        memcpy(&a, &x, sizeof a);
        memcpy(&b, &v, sizeof b);
        b = ((a >> 3) & 1) ? b + 1 : b - 1;
        memcpy(&v, &b, sizeof v);
    }
    return v;
}

/* polynomial_flir (soap.cpp:450-492): the modified-spherical-Bessel overlap of
 * a Gaussian at distance r with each quadrature node, by the reference's
 * downward-stable recurrence clamped at zero; values [(L+1)][Q]. */
static void polynomial_flir(const soap_plan* plan, double radius, double* values) {
    const int Q = plan->grid_size, L = plan->l_max;
    const double eta = plan->eta;
    for (int i = 0; i < (L + 1) * Q; ++i) values[i] = 0.0;
    for (int q = 0; q < Q; ++q) {
        const double radial = plan->grid[q];
        if (radius <= 1e-14) {
            values[q] = flir_exp(-eta * (radial * radial));
            continue;
        }
        const double prefactor = 0.25 / (eta * radius * radial);
        const double minus = flir_exp(-eta * (radial - radius) * (radial - radius));
        const double plus = flir_exp(-eta * (radial + radius) * (radial + radius));
        values[q] = prefactor * (minus - plus);
        if (L >= 1) values[Q + q] = prefactor * (minus + plus - 2.0 * values[q]);
        for (int l = 2; l <= L; ++l) {
            const double v = values[(l - 2) * Q + q] - prefactor * (4.0 * l - 2.0) * values[(l - 1) * Q + q];
            values[l * Q + q] = v > 0.0 ? v : 0.0;
        }
    }
}

/* calculate_coefficients (soap.cpp:701-931) for one centre of one structure. */
static void center_coefficients(const soap_plan* plan, const int* atom_types, int64_t local,
                                const pair_list* pairs, int64_t pair_begin, int64_t pair_end,
                                int64_t structure_begin_index, oreal* coefficients,
                                oreal* scratch) {
    const int S = plan->n_species, n = plan->n_max, L = plan->l_max, H = plan->harmonics;
    const int w = plan->width;
    const int64_t count = pair_end - pair_begin;
    const int pooled = plan->compression == 1;  /* mu2: one density over all species */
    const int CT = pooled ? 1 : S;
    memset(coefficients, 0, sizeof(oreal) * (size_t)CT * n * H);
    /* scratch layout */
    int64_t* order = (int64_t*)scratch;
    oreal* harm = scratch + count;                  /* [count][H] */
    oreal* weight = harm + count * H;               /* [count] */
    oreal* real = weight + count;
    oreal* imag = real + w * w;
    oreal* hs = imag + w * w;                       /* [2L+1] */
    int64_t type_offsets[65];
    int64_t cursor[64];
    for (int t = 0; t <= S; ++t) type_offsets[t] = 0;
    if (pooled) {
        /* graph order, one type range (soap.cpp:716-737) */
        type_offsets[1] = count;
        for (int64_t i = 0; i < count; ++i) order[i] = pair_begin + i;
    } else {
        for (int64_t i = 0; i < count; ++i)
            ++type_offsets[atom_types[pairs->atoms[pair_begin + i] - structure_begin_index] + 1];
        for (int t = 0; t < S; ++t) type_offsets[t + 1] += type_offsets[t];
        for (int t = 0; t < S; ++t) cursor[t] = type_offsets[t];
        for (int64_t i = 0; i < count; ++i) {
            const int t = atom_types[pairs->atoms[pair_begin + i] - structure_begin_index];
            order[cursor[t]++] = pair_begin + i;
        }
    }
    for (int64_t j = 0; j < count; ++j) {
        const int64_t p = order[j];
        const double* d = pairs->displacements + 3 * p;
        const oreal x = d[0], y = d[1], z = d[2];
        solid_harmonics(plan, x, y, z, x * x + y * y + z * z, real, imag, harm + j * H);
    }
    for (int64_t j = 0; j < count; ++j) {
        /* NeighborView::exact_self (neighbor.cpp:683-689): the centre itself, image 0 */
        const int64_t p = order[j];
        const int32_t* sh = pairs->shifts + 3 * p;
        const int self = pairs->atoms[p] - structure_begin_index == local && sh[0] == 0 && sh[1] == 0 && sh[2] == 0;
        const int type = atom_types[pairs->atoms[p] - structure_begin_index];
        weight[j] = soap_weight(plan, sqrt(pairs->distance2[p]), self, type);
    }
    if (plan->radial_basis == 1) {
        /* soap.cpp:799-857: integrand[type][lm][q] accumulated over the
         * neighbours, then projected onto the weighted basis values. */
        const int Q = plan->grid_size;
        double* integrand = calloc((size_t)CT * H * Q, sizeof(double));
        double* flir = malloc(sizeof(double) * (size_t)(L + 1) * Q);
        for (int t = 0; t < CT; ++t) {
            for (int64_t j = type_offsets[t]; j < type_offsets[t + 1]; ++j) {
                const double radius = sqrt(pairs->distance2[order[j]]);
                polynomial_flir(plan, radius, flir);
                const double inverse = radius <= 1e-14 ? 0.0 : 1.0 / radius;
                double inverse_power = 1.0;
                for (int l = 0; l <= L; ++l) {
                    const double scale = radius <= 1e-14 ? (l == 0 ? 4.0 * OR_PI * weight[j] : 0.0)
                                                         : 4.0 * OR_PI * inverse_power * weight[j];
                    for (int m = 0; m < 2 * l + 1; ++m) {
                        const double factor = scale * harm[j * H + l * l + m];
                        double* target = integrand + ((size_t)t * H + l * l + m) * Q;
                        for (int q = 0; q < Q; ++q) target[q] += factor * flir[l * Q + q];
                    }
                    inverse_power *= inverse;
                }
            }
            for (int l = 0; l <= L; ++l)
                for (int nn = 0; nn < n; ++nn)
                    for (int m = 0; m < 2 * l + 1; ++m) {
                        const double* source = integrand + ((size_t)t * H + l * l + m) * Q;
                        double sum = 0.0;
                        for (int q = 0; q < Q; ++q) sum += source[q] * plan->weighted_values[q * n + nn];
                        coefficients[(t * n + nn) * H + l * l + m] += sum;
                    }
        }
        free(integrand);
        free(flir);
        return;
    }
    for (int t = 0; t < CT; ++t) {
        for (int l = 0; l <= L; ++l) {
            const int off = l * l, mc = 2 * l + 1;
            for (int k = 0; k < n; ++k) {
                const int ri = l * n + k;
                for (int m = 0; m < mc; ++m) hs[m] = 0.0;
                for (int64_t j = type_offsets[t]; j < type_offsets[t + 1]; ++j) {
                    const oreal radial = plan->radial_prefactors[ri]
                                         * OEXP(-(oreal)plan->radial_exponents[ri] * pairs->distance2[order[j]]);
                    for (int m = 0; m < mc; ++m) hs[m] += radial * harm[j * H + off + m] * weight[j];
                }
                for (int nn = 0; nn < n; ++nn) {
                    const double beta = plan->betas[(l * n + nn) * n + k];
                    oreal* dest = coefficients + (t * n + nn) * H + off;
                    for (int m = 0; m < mc; ++m) dest[m] += plan->soap_scale * beta * hs[m];
                }
            }
        }
    }
}

/* power spectrum in every compression layout (soap.cpp:933-1017) */
static void power_spectrum(const soap_plan* plan, const oreal* c, oreal* out) {
    const int S = plan->n_species, n = plan->n_max, L = plan->l_max, H = plan->harmonics;
    int64_t f = 0;
    if (plan->compression == 1) { /* mu2: one pooled density, l -> n1 -> n2 >= n1 */
        for (int l = 0; l <= L; ++l)
            for (int n1 = 0; n1 < n; ++n1)
                for (int n2 = n1; n2 < n; ++n2) {
                    oreal sum = 0.0;
                    for (int m = 0; m < 2 * l + 1; ++m) sum += c[n1 * H + l * l + m] * c[n2 * H + l * l + m];
                    out[f++] = plan->power_prefactors[l] * sum;
                }
        return;
    }
    if (plan->compression == 2) { /* mu1nu1: species x species-summed density, all n2 */
        oreal* summed = calloc((size_t)n * H, sizeof(oreal));
        for (int t = 0; t < S; ++t)
            for (int k = 0; k < n; ++k)
                for (int i = 0; i < H; ++i) summed[k * H + i] += c[(t * n + k) * H + i];
        for (int t = 0; t < S; ++t)
            for (int l = 0; l <= L; ++l)
                for (int n1 = 0; n1 < n; ++n1)
                    for (int n2 = 0; n2 < n; ++n2) {
                        oreal sum = 0.0;
                        for (int m = 0; m < 2 * l + 1; ++m)
                            sum += c[(t * n + n1) * H + l * l + m] * summed[n2 * H + l * l + m];
                        out[f++] = plan->power_prefactors[l] * sum;
                    }
        free(summed);
        return;
    }
    if (plan->compression == 3) { /* crossover: same-species pairs, l -> n1 -> n2 >= n1 */
        for (int t = 0; t < S; ++t)
            for (int l = 0; l <= L; ++l)
                for (int n1 = 0; n1 < n; ++n1)
                    for (int n2 = n1; n2 < n; ++n2) {
                        oreal sum = 0.0;
                        for (int m = 0; m < 2 * l + 1; ++m)
                            sum += c[(t * n + n1) * H + l * l + m] * c[(t * n + n2) * H + l * l + m];
                        out[f++] = plan->power_prefactors[l] * sum;
                    }
        return;
    }
    for (int t1 = 0; t1 < S; ++t1)
        for (int t2 = t1; t2 < S; ++t2)
            for (int l = 0; l <= L; ++l) {
                const double pref = plan->power_prefactors[l];
                for (int n1 = 0; n1 < n; ++n1)
                    for (int n2 = (t1 == t2 ? n1 : 0); n2 < n; ++n2) {
                        const oreal* a = c + (t1 * n + n1) * H + l * l;
                        const oreal* b = c + (t2 * n + n2) * H + l * l;
                        oreal sum = 0.0;
                        for (int m = 0; m < 2 * l + 1; ++m) sum += a[m] * b[m];
                        out[f++] = pref * sum;
                    }
            }
}

int64_t oracle_soap_feature_count_ex(int n_species, int n_max, int l_max, int compression) {
    const int64_t W = l_max + 1, n = n_max, S = n_species;
    if (compression == 1) return n * (n + 1) / 2 * W;
    if (compression == 2) return S * n * n * W;
    if (compression == 3) return S * n * (n + 1) / 2 * W;
    return (S * n) * (S * n + 1) / 2 * W;
}

int64_t oracle_soap_feature_count(int n_species, int n_max, int l_max) {
    return oracle_soap_feature_count_ex(n_species, n_max, l_max, 0);
}

/*
 * compute_soap (soap.cpp:1149-1246), GTO basis, compression off.
 * average: 0 off (rows = atoms), 1 inner, 2 outer (rows = structures).
 * species_weights may be NULL (all 1.0).  out is fp64 (rows, F).
 */
int oracle_soap_compute_rbf(const int32_t* numbers, const double* positions, const double* cells,
                            const int32_t* pbc, const int64_t* offsets, int64_t structures,
                            const int32_t* species, int n_species, const double* species_weights,
                            double r_cut, int n_max, int l_max, double sigma, const double* alphas,
                            const double* betas, int average, int compression, int weighting_function,
                            int weighting_has_w0, double weighting_r0, double weighting_c, double weighting_d,
                            double weighting_m, double weighting_w0, int radial_basis, int grid_size,
                            const double* grid, const double* grid_weights, const double* grid_values,
                            int num_threads, double* out) {
    if (validate_batch(numbers, positions, cells, pbc, offsets, structures)) return 1;
    if (!isfinite(r_cut) || !isfinite(sigma) || r_cut <= 0.0 || sigma <= 0.0 || n_max < 1 || l_max < 0
        || l_max > 20 || n_species < 1 || n_species > 64 || average < 0 || average > 2 || compression < 0
        || compression > 3 || weighting_function < 0 || weighting_function > 3 || radial_basis < 0
        || radial_basis > 1)
        return fail("invalid SOAP parameters");
    if (radial_basis == 1 && (grid_size < 2 || !grid || !grid_weights || !grid_values))
        return fail("invalid SOAP polynomial radial basis size");
    soap_plan plan;
    plan.radial_basis = radial_basis;
    plan.grid_size = radial_basis == 1 ? grid_size : 0;
    plan.grid = grid;
    plan.eta = 1.0 / (2.0 * sigma * sigma);
    plan.weighted_values = NULL;
    if (radial_basis == 1) {
        plan.weighted_values = malloc(sizeof(double) * (size_t)grid_size * n_max);
        for (int q = 0; q < grid_size; ++q) {
            const double quadrature = grid_weights[q] * grid[q] * grid[q];
            for (int k = 0; k < n_max; ++k)
                plan.weighted_values[q * n_max + k] = quadrature * grid_values[k * grid_size + q];
        }
    }
    plan.compression = compression;
    plan.weighting_function = weighting_function;
    plan.weighting_has_w0 = weighting_has_w0;
    plan.weighting_r0 = weighting_r0;
    plan.weighting_c = weighting_c;
    plan.weighting_d = weighting_d;
    plan.weighting_m = weighting_m;
    plan.weighting_w0 = weighting_w0;
    plan.n_species = n_species;
    plan.n_max = n_max;
    plan.l_max = l_max;
    plan.width = l_max + 1;
    plan.harmonics = (l_max + 1) * (l_max + 1);
    plan.species = species;
    double* ones = malloc(sizeof(double) * (size_t)n_species);
    for (int t = 0; t < n_species; ++t) ones[t] = species_weights ? species_weights[t] : 1.0;
    plan.species_weights = ones;
    plan.betas = betas;
    plan.soap_scale = OR_PI * sqrt(OR_PI);
    const int w = l_max + 1;
    plan.power_prefactors = malloc(sizeof(double) * w);
    plan.normalization = calloc((size_t)w * w, sizeof(double));
    plan.radial_prefactors = malloc(sizeof(double) * w * n_max);
    plan.radial_exponents = malloc(sizeof(double) * w * n_max);
    for (int l = 0; l <= l_max; ++l) {
        plan.power_prefactors[l] = OR_PI * sqrt(8.0 / (2.0 * l + 1.0));
        for (int m = 0; m <= l; ++m)
            plan.normalization[l * w + m] =
                sqrt((2.0 * l + 1.0) / (4.0 * OR_PI) * exp(lgamma(l - m + 1.0) - lgamma(l + m + 1.0)));
    }
    const double eta = 1.0 / (2.0 * sigma * sigma);
    double eta_power = 1.0;
    for (int l = 0; l <= l_max && radial_basis == 0; ++l) {
        if (l > 0) eta_power *= eta;
        for (int k = 0; k < n_max; ++k) {
            const int i = l * n_max + k;
            const double alpha = alphas[i];
            const double denominator = alpha + eta;
            plan.radial_prefactors[i] = eta_power * pow(denominator, -l - 1.5);
            plan.radial_exponents[i] = alpha * eta / denominator;
        }
    }
    const double cutoff = r_cut + sigma * sqrt(-2.0 * log(1e-3));
    const int64_t F = oracle_soap_feature_count_ex(n_species, n_max, l_max, compression);
    const int64_t csize = (int64_t)(compression == 1 ? 1 : n_species) * n_max * plan.harmonics;
    int status = 0;
#ifdef _OPENMP
    const int threads = num_threads > 0 ? num_threads : omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads) reduction(| : status)
#endif
    for (int64_t s = 0; s < structures; ++s) {
        if (status) continue;
        const int64_t begin = offsets[s], end = offsets[s + 1], atoms = end - begin;
        pair_list pairs = {0};
        int64_t* counts = malloc(sizeof(int64_t) * ((size_t)atoms + 1));
        int* types = malloc(sizeof(int) * ((size_t)atoms + 1));
        oreal* coefficients = malloc(sizeof(oreal) * (size_t)csize);
        oreal* accumulated = calloc((size_t)csize, sizeof(oreal));
        oreal* power = malloc(sizeof(oreal) * (size_t)F);
        oreal* power_sum = calloc((size_t)F, sizeof(oreal));
        int local_status = structure_graph(positions, cells + 9 * s, pbc + 3 * s, begin, end, cutoff,
                                           0, NULL, 0, &pairs, counts);
        for (int64_t i = 0; i < atoms && !local_status; ++i) {
            types[i] = species_type(&plan, numbers[begin + i]);
            if (types[i] < 0) local_status = fail("batch contains an atomic number outside calculator species");
        }
        int64_t max_count = 0;
        for (int64_t i = 0; i < atoms && !local_status; ++i)
            if (counts[i + 1] - counts[i] > max_count) max_count = counts[i + 1] - counts[i];
        oreal* scratch = malloc(sizeof(oreal) * (size_t)(max_count * (plan.harmonics + 3) + 4 * w * w + 64));
        for (int64_t i = 0; i < atoms && !local_status; ++i) {
            center_coefficients(&plan, types, i, &pairs, counts[i], counts[i + 1], 0, coefficients, scratch);
            if (average == 0) {
                power_spectrum(&plan, coefficients, power);
                for (int64_t k = 0; k < F; ++k) out[(begin + i) * F + k] = (double)power[k];
            } else if (average == 1) {
                for (int64_t k = 0; k < csize; ++k) accumulated[k] += coefficients[k];
            } else {
                power_spectrum(&plan, coefficients, power);
                for (int64_t k = 0; k < F; ++k) power_sum[k] += power[k];
            }
        }
        if (!local_status && average == 1) {
            if (atoms > 0) {
                const double inverse = 1.0 / (double)atoms;
                for (int64_t k = 0; k < csize; ++k) accumulated[k] *= inverse;
            }
            power_spectrum(&plan, accumulated, power);
            for (int64_t k = 0; k < F; ++k) out[s * F + k] = (double)power[k];
        } else if (!local_status && average == 2) {
            for (int64_t k = 0; k < F; ++k) out[s * F + k] = atoms > 0 ? (double)(power_sum[k] / (double)atoms) : 0.0;
        }
        free(scratch);
        free(counts);
        free(types);
        free(coefficients);
        free(accumulated);
        free(power);
        free(power_sum);
        pair_free(&pairs);
        status |= local_status;
    }
    free(ones);
    free(plan.power_prefactors);
    free(plan.normalization);
    free(plan.radial_prefactors);
    free(plan.radial_exponents);
    free(plan.weighted_values);
    return status;
}

int oracle_soap_compute_ex(const int32_t* numbers, const double* positions, const double* cells,
                           const int32_t* pbc, const int64_t* offsets, int64_t structures,
                           const int32_t* species, int n_species, const double* species_weights,
                           double r_cut, int n_max, int l_max, double sigma, const double* alphas,
                           const double* betas, int average, int compression, int weighting_function,
                           int weighting_has_w0, double weighting_r0, double weighting_c, double weighting_d,
                           double weighting_m, double weighting_w0, int num_threads, double* out) {
    return oracle_soap_compute_rbf(numbers, positions, cells, pbc, offsets, structures, species, n_species,
                                   species_weights, r_cut, n_max, l_max, sigma, alphas, betas, average, compression,
                                   weighting_function, weighting_has_w0, weighting_r0, weighting_c, weighting_d,
                                   weighting_m, weighting_w0, 0, 0, NULL, NULL, NULL, num_threads, out);
}

/* compute_soap with compression off and no weighting function. */
int oracle_soap_compute(const int32_t* numbers, const double* positions, const double* cells,
                        const int32_t* pbc, const int64_t* offsets, int64_t structures,
                        const int32_t* species, int n_species, const double* species_weights,
                        double r_cut, int n_max, int l_max, double sigma, const double* alphas,
                        const double* betas, int average, int num_threads, double* out) {
    return oracle_soap_compute_ex(numbers, positions, cells, pbc, offsets, structures, species, n_species,
                                  species_weights, r_cut, n_max, l_max, sigma, alphas, betas, average, 0, 0, 0, 1.0,
                                  1.0, 0.0, 1.0, 1.0, num_threads, out);
}

/*
 * Rows of the average-"off" feature matrix for selected atoms only (global
 * indices `rows`, any order): the same per-centre arithmetic as
 * oracle_soap_compute, with the neighbour query restricted to the requested
 * centres.  Lets tests check sampled rows of full-size structures.
 */
int oracle_soap_rows(const int32_t* numbers, const double* positions, const double* cells,
                     const int32_t* pbc, const int64_t* offsets, int64_t structures,
                     const int32_t* species, int n_species, const double* species_weights,
                     double r_cut, int n_max, int l_max, double sigma, const double* alphas,
                     const double* betas, const int64_t* rows, int64_t n_rows, double* out) {
    if (validate_batch(numbers, positions, cells, pbc, offsets, structures)) return 1;
    if (!isfinite(r_cut) || !isfinite(sigma) || r_cut <= 0.0 || sigma <= 0.0 || n_max < 1 || l_max < 0
        || l_max > 20 || n_species < 1 || n_species > 64)
        return fail("invalid SOAP parameters");
    soap_plan plan;
    plan.compression = 0;
    plan.weighting_function = 0;
    plan.weighting_has_w0 = 0;
    plan.weighting_r0 = plan.weighting_c = plan.weighting_m = plan.weighting_w0 = 1.0;
    plan.weighting_d = 0.0;
    plan.radial_basis = 0;
    plan.grid_size = 0;
    plan.grid = NULL;
    plan.weighted_values = NULL;
    plan.eta = 1.0 / (2.0 * sigma * sigma);
    plan.n_species = n_species;
    plan.n_max = n_max;
    plan.l_max = l_max;
    plan.width = l_max + 1;
    plan.harmonics = (l_max + 1) * (l_max + 1);
    plan.species = species;
    double* weights = malloc(sizeof(double) * (size_t)n_species);
    for (int t = 0; t < n_species; ++t) weights[t] = species_weights ? species_weights[t] : 1.0;
    plan.species_weights = weights;
    plan.betas = betas;
    plan.soap_scale = OR_PI * sqrt(OR_PI);
    const int w = l_max + 1;
    plan.power_prefactors = malloc(sizeof(double) * w);
    plan.normalization = calloc((size_t)w * w, sizeof(double));
    plan.radial_prefactors = malloc(sizeof(double) * w * n_max);
    plan.radial_exponents = malloc(sizeof(double) * w * n_max);
    for (int l = 0; l <= l_max; ++l) {
        plan.power_prefactors[l] = OR_PI * sqrt(8.0 / (2.0 * l + 1.0));
        for (int m = 0; m <= l; ++m)
            plan.normalization[l * w + m] =
                sqrt((2.0 * l + 1.0) / (4.0 * OR_PI) * exp(lgamma(l - m + 1.0) - lgamma(l + m + 1.0)));
    }
    const double eta = 1.0 / (2.0 * sigma * sigma);
    double eta_power = 1.0;
    for (int l = 0; l <= l_max; ++l) {
        if (l > 0) eta_power *= eta;
        for (int k = 0; k < n_max; ++k) {
            const int i = l * n_max + k;
            const double denominator = alphas[i] + eta;
            plan.radial_prefactors[i] = eta_power * pow(denominator, -l - 1.5);
            plan.radial_exponents[i] = alphas[i] * eta / denominator;
        }
    }
    const double cutoff = r_cut + sigma * sqrt(-2.0 * log(1e-3));
    const int64_t F = oracle_soap_feature_count(n_species, n_max, l_max);
    const int64_t csize = (int64_t)n_species * n_max * plan.harmonics;
    int status = 0;
    for (int64_t s = 0; s < structures && !status; ++s) {
        const int64_t begin = offsets[s], end = offsets[s + 1], atoms = end - begin;
        int64_t wanted = 0;
        for (int64_t r = 0; r < n_rows; ++r) wanted += rows[r] >= begin && rows[r] < end;
        if (!wanted) continue;
        int64_t* subset = malloc(sizeof(int64_t) * (size_t)wanted);
        int64_t* slot = malloc(sizeof(int64_t) * (size_t)wanted);
        int64_t q = 0;
        for (int64_t r = 0; r < n_rows; ++r)
            if (rows[r] >= begin && rows[r] < end) {
                subset[q] = rows[r] - begin;
                slot[q++] = r;
            }
        int* types = malloc(sizeof(int) * ((size_t)atoms + 1));
        for (int64_t i = 0; i < atoms && !status; ++i) {
            types[i] = species_type(&plan, numbers[begin + i]);
            if (types[i] < 0) status = fail("batch contains an atomic number outside calculator species");
        }
        pair_list pairs = {0};
        int64_t* counts = malloc(sizeof(int64_t) * ((size_t)wanted + 1));
        if (!status)
            status = structure_graph(positions, cells + 9 * s, pbc + 3 * s, begin, end, cutoff, 0, subset, wanted,
                                     &pairs, counts);
        int64_t max_count = 0;
        for (int64_t i = 0; i < wanted && !status; ++i)
            if (counts[i + 1] - counts[i] > max_count) max_count = counts[i + 1] - counts[i];
        oreal* coefficients = malloc(sizeof(oreal) * (size_t)csize);
        oreal* power = malloc(sizeof(oreal) * (size_t)F);
        oreal* scratch = malloc(sizeof(oreal) * (size_t)(max_count * (plan.harmonics + 3) + 4 * w * w + 64));
        for (int64_t i = 0; i < wanted && !status; ++i) {
            center_coefficients(&plan, types, subset[i], &pairs, counts[i], counts[i + 1], 0, coefficients, scratch);
            power_spectrum(&plan, coefficients, power);
            for (int64_t k = 0; k < F; ++k) out[slot[i] * F + k] = (double)power[k];
        }
        free(power);
        free(scratch);
        free(coefficients);
        free(counts);
        pair_free(&pairs);
        free(types);
        free(subset);
        free(slot);
    }
    free(weights);
    free(plan.power_prefactors);
    free(plan.normalization);
    free(plan.radial_prefactors);
    free(plan.radial_exponents);
    return status;
}
