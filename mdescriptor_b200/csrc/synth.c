/*
 * Seeded synthetic periodic cells for the large SOAP benchmark batches
 * (host code, C99 + OpenMP).  Benchmark/test input generation only: nothing
 * on the descriptor path calls it.
 *
 * Structure s of a batch draws from its own counter-based stream, seeded by
 * (seed, s) alone, so any contiguous range of a batch's structures can be
 * generated on its own (each rank of a sharded run makes only its slice) and
 * equals the same range of the whole batch.  Per structure: `atoms` positions
 * uniform in the cubic cell [0, side)^3, each redrawn until its minimum-image
 * distance to every earlier atom of the structure is >= d_min; then one
 * species per atom, drawn with the given weights.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

/* splitmix64 (Steele, Lea, Flood, "Fast splittable pseudorandom number
 * generators", OOPSLA 2014). */
static inline uint64_t next_u64(uint64_t* state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Uniform double in [0, 1) from the top 53 bits. */
static inline double next_unit(uint64_t* state) { return (double)(next_u64(state) >> 11) * 0x1.0p-53; }

static uint64_t structure_state(uint64_t seed, int64_t structure) {
    uint64_t s = seed ^ 0x6A09E667F3BCC909ull;
    (void)next_u64(&s);
    s ^= (uint64_t)structure * 0xD1342543DE82EF95ull + 0x2545F4914F6CDD1Dull;
    (void)next_u64(&s);
    return s;
}

/* Structures [first, first + count) of the batch; numbers int32[count*atoms],
 * positions float64[count*atoms*3].  Returns 0, or -1 when a structure needed
 * more than max_tries draws for one atom (cell too dense for d_min). */
int mdsynth_cubic(uint64_t seed, int64_t first, int64_t count, int32_t atoms, double side, double d_min,
                  int32_t n_species, const int32_t* species, const double* weights, int32_t* numbers,
                  double* positions, int64_t max_tries) {
    const double d2_min = d_min * d_min, inv = 1.0 / side;
    double total = 0.0;
    for (int32_t i = 0; i < n_species; ++i) total += weights[i];
    int failed = 0;
#pragma omp parallel for schedule(dynamic, 16) reduction(| : failed)
    for (int64_t i = 0; i < count; ++i) {
        uint64_t state = structure_state(seed, first + i);
        double* x = positions + (size_t)i * (size_t)atoms * 3;
        for (int32_t k = 0; k < atoms && !failed; ++k) {
            int64_t tries = 0;
            for (;;) {
                const double cx = side * next_unit(&state), cy = side * next_unit(&state),
                             cz = side * next_unit(&state);
                int ok = 1;
                for (int32_t j = 0; j < k && ok; ++j) {
                    double dx = x[3 * j] - cx, dy = x[3 * j + 1] - cy, dz = x[3 * j + 2] - cz;
                    dx -= side * nearbyint(dx * inv);
                    dy -= side * nearbyint(dy * inv);
                    dz -= side * nearbyint(dz * inv);
                    ok = dx * dx + dy * dy + dz * dz >= d2_min;
                }
                if (ok) {
                    x[3 * k] = cx;
                    x[3 * k + 1] = cy;
                    x[3 * k + 2] = cz;
                    break;
                }
                if (++tries >= max_tries) {
                    failed = 1;
                    break;
                }
            }
        }
        int32_t* z = numbers + (size_t)i * (size_t)atoms;
        for (int32_t k = 0; k < atoms; ++k) {
            const double u = total * next_unit(&state);
            double acc = 0.0;
            int32_t pick = n_species - 1;
            for (int32_t t = 0; t < n_species; ++t) {
                acc += weights[t];
                if (u < acc) {
                    pick = t;
                    break;
                }
            }
            z[k] = species[pick];
        }
    }
    return failed ? -1 : 0;
}
