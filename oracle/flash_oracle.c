/*
 * CPU oracle for the flash-attention forward path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is the parity checker for the sm_100a kernel in
 * not-cute-zig_b200/csrc.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load it.  The product library never links or calls it.
 *
 * It restates, in plain C, the reference's CPU attention:
 *   - computeFlashReferenceOne    src/main.zig:1271-1307
 *   - computeFlashReferenceSlices src/main.zig:1242-1269
 *   - fillFlashInput              src/main.zig:1207-1211
 *   - the benchmark input pattern src/main.zig:782-791 (mod 11 / 13 / 17)
 * The operation order is kept: an f32 dot product in ascending k, then
 * `score *= scale`; -inf for future keys under causal masking; a running row
 * max; weights exp(score - max) summed in ascending key order; then, for each
 * output column, acc += (weight / row_sum) * v in ascending key order.
 *
 * Extension (not expressible in the reference API): per-row element strides
 * for Q/K/V/O.  With row_stride == head_dim this is exactly the reference.
 *
 * Also here: a seeded generator (splitmix64 -> uniform -> Box-Muller), so
 * synthetic inputs are bit-identical on every machine.  The kernel and the
 * oracle both read the same f16 bits.
 *
 * Build: gcc -O2 -fno-fast-math -fopenmp -shared -fPIC (see oracle/build.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef uint16_t f16bits;

static inline float h2f(f16bits h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

/* bf16 bits -> f32: the upper half of the f32 bit pattern (exact). */
static inline float b2f(f16bits h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* f32 -> bf16 bits, round to nearest even (NaN kept quiet). */
static inline f16bits f2b(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0u) return (f16bits)((u >> 16) | 0x40u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (f16bits)(u >> 16);
}

static inline f16bits f2h(float f) {
    _Float16 v = (_Float16)f; /* round to nearest even */
    f16bits h;
    memcpy(&h, &v, 2);
    return h;
}

/* Restates computeFlashReferenceOne (src/main.zig:1271-1307) for one
 * batch x head slice; `scores` is caller-provided scratch of seq_len floats.
 * When `mag` is given it also receives, per output element, sum_k w_k |v_k|
 * with the same normalised weights w_k: the magnitude that bounds the effect
 * of rounding the weights (the reference GPU kernels round P to f16,
 * src/flash_h64_bn32.zig:185) on that output, |sum_k d_k w_k v_k| <= u * mag
 * when every |d_k| <= u.  It is test bookkeeping, not part of the restated
 * algorithm. */
static void flash_one_row(size_t seq_len, size_t head_dim, size_t row, const f16bits *q,
                          size_t q_row, const f16bits *k, size_t k_row, const f16bits *v,
                          size_t v_row, float *o, float *mag, size_t o_row, float scale, uint32_t causal,
                          float *scores, int bf16) {
    float (*const in)(f16bits) = bf16 ? b2f : h2f; /* Q/K/V element type */
    float row_max = -INFINITY;
    for (size_t key = 0; key < seq_len; ++key) {
        if (causal != 0 && key > row) {
            scores[key] = -INFINITY; /* main.zig:1277-1278 */
        } else {
            float score = 0.0f;
            for (size_t kk = 0; kk < head_dim; ++kk) /* main.zig:1281-1284 */
                score += in(q[row * q_row + kk]) * in(k[key * k_row + kk]);
            score *= scale; /* main.zig:1285 */
            scores[key] = score;
            row_max = fmaxf(row_max, score);
        }
    }
    float row_sum = 0.0f;
    for (size_t key = 0; key < seq_len; ++key) { /* main.zig:1291-1296 */
        const float weight = scores[key] == -INFINITY ? 0.0f : expf(scores[key] - row_max);
        scores[key] = weight;
        row_sum += weight;
    }
    for (size_t col = 0; col < head_dim; ++col) { /* main.zig:1298-1305 */
        float acc = 0.0f;
        for (size_t key = 0; key < seq_len; ++key) {
            const float weight = scores[key] / row_sum;
            acc += weight * in(v[key * v_row + col]);
        }
        o[row * o_row + col] = acc;
    }
    if (mag != NULL) {
        for (size_t col = 0; col < head_dim; ++col) {
            double acc = 0.0;
            for (size_t key = 0; key < seq_len; ++key)
                acc += (double)(scores[key] / row_sum) * fabs((double)in(v[key * v_row + col]));
            mag[row * o_row + col] = (float)acc;
        }
    }
}

/*
 * All slices (computeFlashReferenceSlices, src/main.zig:1242-1269) with the
 * row-stride extension.  Slices and rows are independent, so (slice, row)
 * pairs are spread over `nthreads` OpenMP threads (<= 0: all available).
 * Rows `row_begin..row_end` of every slice are computed (the full range is
 * 0..seq_len); the CPU baseline uses a subrange as its bounded sample.
 * Output elements outside the active rows are not touched.
 */
static void oracle_flash(size_t batch_heads, size_t seq_len, size_t head_dim, const f16bits *q,
                         size_t q_stride, size_t q_row, const f16bits *k, size_t k_stride,
                         size_t k_row, const f16bits *v, size_t v_stride, size_t v_row, float *o,
                         float *mag, size_t o_stride, size_t o_row, float scale, uint32_t causal,
                         size_t row_begin, size_t row_end, int nthreads, int bf16) {
    if (row_end > seq_len) row_end = seq_len;
    if (row_begin >= row_end || batch_heads == 0) return;
    const size_t rows = row_end - row_begin;
    const long long total = (long long)(batch_heads * rows);
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
    (void)nthreads;
#endif
#pragma omp parallel num_threads(nthreads)
    {
        float *scores = (float *)malloc(seq_len * sizeof(float));
#pragma omp for schedule(dynamic, 4)
        for (long long i = 0; i < total; ++i) {
            const size_t slice = (size_t)i / rows;
            const size_t row = row_begin + (size_t)i % rows;
            flash_one_row(seq_len, head_dim, row, q + slice * q_stride, q_row,
                          k + slice * k_stride, k_row, v + slice * v_stride, v_row,
                          o + slice * o_stride, mag != NULL ? mag + slice * o_stride : NULL, o_row, scale,
                          causal, scores, bf16);
        }
        free(scores);
    }
}

void ncz_oracle_flash(size_t batch_heads, size_t seq_len, size_t head_dim, const f16bits *q,
                      size_t q_stride, size_t q_row, const f16bits *k, size_t k_stride,
                      size_t k_row, const f16bits *v, size_t v_stride, size_t v_row, float *o,
                      size_t o_stride, size_t o_row, float scale, uint32_t causal,
                      size_t row_begin, size_t row_end, int nthreads) {
    oracle_flash(batch_heads, seq_len, head_dim, q, q_stride, q_row, k, k_stride, k_row, v, v_stride,
                 v_row, o, NULL, o_stride, o_row, scale, causal, row_begin, row_end, nthreads, 0);
}

/* ncz_oracle_flash plus, in `mag` (laid out like o), the per-element magnitude
 * sum_k w_k |v_k| (see flash_one_row); bf16 != 0 reads bf16 Q/K/V. */
void ncz_oracle_flash_mag(size_t batch_heads, size_t seq_len, size_t head_dim, const f16bits *q,
                          size_t q_stride, size_t q_row, const f16bits *k, size_t k_stride,
                          size_t k_row, const f16bits *v, size_t v_stride, size_t v_row, float *o,
                          float *mag, size_t o_stride, size_t o_row, float scale, uint32_t causal,
                          size_t row_begin, size_t row_end, int nthreads, int bf16) {
    oracle_flash(batch_heads, seq_len, head_dim, q, q_stride, q_row, k, k_stride, k_row, v, v_stride,
                 v_row, o, mag, o_stride, o_row, scale, causal, row_begin, row_end, nthreads, bf16 != 0);
}

/* The same maths on bf16 Q/K/V (the reference has f16 only; this extends the
 * restatement to the bf16 input path of the kernel). */
void ncz_oracle_flash_bf16(size_t batch_heads, size_t seq_len, size_t head_dim, const f16bits *q,
                           size_t q_stride, size_t q_row, const f16bits *k, size_t k_stride,
                           size_t k_row, const f16bits *v, size_t v_stride, size_t v_row, float *o,
                           size_t o_stride, size_t o_row, float scale, uint32_t causal,
                           size_t row_begin, size_t row_end, int nthreads) {
    oracle_flash(batch_heads, seq_len, head_dim, q, q_stride, q_row, k, k_stride, k_row, v, v_stride,
                 v_row, o, NULL, o_stride, o_row, scale, causal, row_begin, row_end, nthreads, 1);
}

/* fillFlashInput (src/main.zig:1207-1211):
 * data[i] = f16(((i * mul + add) % modulus) * scale); the smoke and compare
 * inputs use modulus 17, the benchmark inputs use 11 / 13 / 17 (main.zig:782-791). */
void ncz_oracle_fill_pattern(f16bits *data, size_t n, size_t mul, size_t add, size_t modulus,
                             float scale) {
    for (size_t i = 0; i < n; ++i)
        data[i] = f2h((float)((i * mul + add) % modulus) * scale);
}

static inline uint64_t splitmix64(uint64_t *state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Uniform double in (0, 1): 53 random bits, offset by half an ulp so 0 never occurs. */
static inline double uniform01(uint64_t *state) {
    return ((double)(splitmix64(state) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

/* The generator is counter based: after c draws from seed the state is
 * seed + c * 0x9E3779B97F4A7C15 (mod 2^64), so any stretch of the stream can
 * be produced on its own, and in parallel, with the same bits. */
#define NCZ_GOLDEN_GAMMA 0x9E3779B97F4A7C15ull

/* Elements first .. first+n-1 of the stream f16(mean + std * N(0,1)): element
 * 2p and 2p+1 are the cos and sin halves of the Box-Muller pair made from
 * draws 2p and 2p+1 of splitmix64(seed). */
static void fill_normal_as(f16bits *data, size_t n, uint64_t seed, size_t first, float mean, float stddev,
                           f16bits (*enc)(float)) {
    const double two_pi = 6.283185307179586476925286766559;
    const size_t end = first + n;
    const size_t p0 = first / 2, p1 = (end + 1) / 2;  /* pairs touched */
    const ptrdiff_t np = (ptrdiff_t)(p1 - p0);
#pragma omp parallel for schedule(static) if (np > 65536)
    for (ptrdiff_t j = 0; j < np; ++j) {
        const size_t pair = p0 + (size_t)j;
        uint64_t state = seed + (uint64_t)(2 * pair) * NCZ_GOLDEN_GAMMA;
        const double u1 = uniform01(&state), u2 = uniform01(&state);
        const double r = sqrt(-2.0 * log(u1));
        const size_t e0 = 2 * pair, e1 = e0 + 1;
        if (e0 >= first && e0 < end) data[e0 - first] = enc((float)(mean + stddev * r * cos(two_pi * u2)));
        if (e1 >= first && e1 < end) data[e1 - first] = enc((float)(mean + stddev * r * sin(two_pi * u2)));
    }
}

void ncz_oracle_fill_normal(f16bits *data, size_t n, uint64_t seed, float mean, float stddev) {
    fill_normal_as(data, n, seed, 0, mean, stddev, f2h);
}

/* ncz_oracle_fill_normal's stream from element `first` on. */
void ncz_oracle_fill_normal_range(f16bits *data, size_t n, uint64_t seed, size_t first, float mean, float stddev) {
    fill_normal_as(data, n, seed, first, mean, stddev, f2h);
}

/* bf16 (round to nearest even) from the same splitmix64 + Box-Muller stream. */
void ncz_oracle_fill_normal_bf16(f16bits *data, size_t n, uint64_t seed, float mean, float stddev) {
    fill_normal_as(data, n, seed, 0, mean, stddev, f2b);
}

/* Elements first .. first+n-1 of f16(U(lo, hi)): element i from draw i. */
void ncz_oracle_fill_uniform_range(f16bits *data, size_t n, uint64_t seed, size_t first, float lo, float hi) {
    const ptrdiff_t nn = (ptrdiff_t)n;
#pragma omp parallel for schedule(static) if (nn > 65536)
    for (ptrdiff_t j = 0; j < nn; ++j) {
        uint64_t state = seed + (uint64_t)(first + (size_t)j) * NCZ_GOLDEN_GAMMA;
        data[j] = f2h((float)(lo + (hi - lo) * uniform01(&state)));
    }
}

void ncz_oracle_fill_uniform(f16bits *data, size_t n, uint64_t seed, float lo, float hi) {
    ncz_oracle_fill_uniform_range(data, n, seed, 0, lo, hi);
}

/* Sets every element of a strided [batch_heads, seq_len, row] view whose
 * column is >= head_dim (the row padding) to `value_bits` (e.g. an f16 NaN).
 * Padding only exists when row_stride > head_dim. */
void ncz_oracle_fill_row_padding(f16bits *data, size_t batch_heads, size_t seq_len,
                                 size_t head_dim, size_t slice_stride, size_t row_stride,
                                 f16bits value_bits) {
    for (size_t b = 0; b < batch_heads; ++b)
        for (size_t r = 0; r < seq_len; ++r)
            for (size_t c = head_dim; c < row_stride; ++c)
                data[b * slice_stride + r * row_stride + c] = value_bits;
}

int ncz_oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
