/*
 * CPU oracle for the BF16 GEMM hot path of kernel_mcts.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library, and only as the checker
 * (or the timed CPU baseline).  The product path never calls it.
 *
 * What it restates (reference paths are relative to the reference project):
 *
 *  - Input stream: src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:92-95
 *    and bf16_input_generator.cu:23-37.  std::mt19937(seed), then
 *    std::uniform_real_distribution<float>(-0.25f, 0.25f), each draw rounded to
 *    BF16 by __float2bfloat16 (round-to-nearest-even).  A (M*K values) is drawn
 *    first, then B (K*N values), from one generator.
 *    mt19937 is the published Mersenne Twister (Matsumoto & Nishimura 1998).
 *    The float draw follows the C++ standard's generate_canonical<float, 24>
 *    with a 32-bit engine: u = float(x) / 2^32, clamped below 1, then
 *    a + u * (b - a).
 *
 *  - GEMM: the root program src/kernel_mcts/benchmarks/kernels/bf16_gemm_root.cu:8-44.
 *    Each C[i,j] is one FP32 accumulator, started at +0, updated by one fused
 *    multiply-add per k in increasing k order (nvcc contracts
 *    `acc += a * b` to FFMA at -O3), over K rounded up to 16 with zero padding,
 *    then rounded once to BF16 (RNE).  A is [M,K] row-major; B is either the
 *    contract's column-major [K,N] (B[j*K + k]) or row-major [K,N] (B[k*N + j]).
 *
 *  - Error check: bf16_gemm_harness.cu:154-164.  maximum and mean absolute
 *    error in double, success iff every output is finite and
 *    |c - ref| <= atol + rtol * |ref|.
 *
 * Parity of this oracle is pinned by tests/golden (inputs from the
 * reference's own compiled generator; outputs of the reference's own root
 * kernel run on a B200).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- mt19937 */

typedef struct {
    uint32_t state[624];
    int index;
} kmcts_mt19937;

static void mt_seed(kmcts_mt19937* mt, uint32_t seed) {
    mt->state[0] = seed;
    for (int i = 1; i < 624; ++i) {
        uint32_t prev = mt->state[i - 1];
        mt->state[i] = 1812433253u * (prev ^ (prev >> 30)) + (uint32_t)i;
    }
    mt->index = 624;
}

static void mt_twist(kmcts_mt19937* mt) {
    for (int i = 0; i < 624; ++i) {
        uint32_t y = (mt->state[i] & 0x80000000u) | (mt->state[(i + 1) % 624] & 0x7fffffffu);
        uint32_t next = mt->state[(i + 397) % 624] ^ (y >> 1);
        if (y & 1u) next ^= 0x9908b0dfu;
        mt->state[i] = next;
    }
    mt->index = 0;
}

static uint32_t mt_next(kmcts_mt19937* mt) {
    if (mt->index >= 624) mt_twist(mt);
    uint32_t y = mt->state[mt->index++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

/* ------------------------------------------------------------- BF16 bits */

uint16_t kmcts_oracle_float_to_bf16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof(bits));
    if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu) != 0u) {
        return 0x7fffu; /* canonical quiet NaN, as __float2bfloat16 produces */
    }
    uint32_t rounding_bias = 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + rounding_bias) >> 16);
}

float kmcts_oracle_bf16_to_float(uint16_t value) {
    uint32_t bits = (uint32_t)value << 16;
    float out;
    memcpy(&out, &bits, sizeof(out));
    return out;
}

/* ---------------------------------------------------------------- inputs */

static float canonical_uniform(kmcts_mt19937* mt) {
    const float range = 4294967296.0f; /* engine max - min + 1 = 2^32 */
    float u = (float)mt_next(mt) / range;
    if (u >= 1.0f) u = nextafterf(1.0f, 0.0f);
    return u;
}

/* Fills A (a_count values) then B (b_count values) from one generator,
 * exactly as the reference harness does.  Outputs are BF16 bit patterns. */
void kmcts_oracle_uniform_inputs(uint32_t seed, size_t a_count, size_t b_count,
                                 uint16_t* a_out, uint16_t* b_out) {
    kmcts_mt19937 mt;
    mt_seed(&mt, seed);
    const float lo = -0.25f, hi = 0.25f;
    for (size_t i = 0; i < a_count; ++i) {
        float u = canonical_uniform(&mt);
        a_out[i] = kmcts_oracle_float_to_bf16(u * (hi - lo) + lo);
    }
    for (size_t i = 0; i < b_count; ++i) {
        float u = canonical_uniform(&mt);
        b_out[i] = kmcts_oracle_float_to_bf16(u * (hi - lo) + lo);
    }
}

/* Raw mt19937 words, used by the tests to check the engine itself. */
void kmcts_oracle_mt19937_words(uint32_t seed, size_t count, uint32_t* out) {
    kmcts_mt19937 mt;
    mt_seed(&mt, seed);
    for (size_t i = 0; i < count; ++i) out[i] = mt_next(&mt);
}

/* ------------------------------------------------------------------ GEMM */

/* Sequential-FMA GEMM with the root program's accumulation order.
 * b_layout 0: B column-major [K,N] (element (k,j) at B[j*K + k]).
 * b_layout 1: B row-major [K,N] (element (k,j) at B[k*N + j]).
 * Returns 0 on success, 1 on bad arguments, 2 on allocation failure. */
int kmcts_oracle_gemm(const uint16_t* A, const uint16_t* B, uint16_t* C,
                      int M, int N, int K, int b_layout) {
    if (M < 0 || N < 0 || K < 0 || (b_layout != 0 && b_layout != 1)) return 1;
    if (M == 0 || N == 0) return 0;
    const int k_padded = (K + 15) / 16 * 16;
    /* Widen once: af[i*K + k], bf[k*N + j] (row-major [K,N]). */
    float* af = (float*)malloc(sizeof(float) * (size_t)M * (size_t)(K ? K : 1));
    float* bf = (float*)malloc(sizeof(float) * (size_t)(K ? K : 1) * (size_t)N);
    if (!af || !bf) {
        free(af);
        free(bf);
        return 2;
    }
    for (size_t i = 0; i < (size_t)M * (size_t)K; ++i) af[i] = kmcts_oracle_bf16_to_float(A[i]);
    for (int k = 0; k < K; ++k) {
        for (int j = 0; j < N; ++j) {
            uint16_t v = b_layout == 0 ? B[(size_t)j * K + k] : B[(size_t)k * N + j];
            bf[(size_t)k * N + j] = kmcts_oracle_bf16_to_float(v);
        }
    }
    enum { ROWS = 32, COLS = 256 };
    const int row_blocks = (M + ROWS - 1) / ROWS;
    const int col_blocks = (N + COLS - 1) / COLS;
#pragma omp parallel for schedule(dynamic)
    for (int block = 0; block < row_blocks * col_blocks; ++block) {
        const int i0 = (block / col_blocks) * ROWS;
        const int j0 = (block % col_blocks) * COLS;
        const int rows = M - i0 < ROWS ? M - i0 : ROWS;
        const int cols = N - j0 < COLS ? N - j0 : COLS;
        float acc[ROWS][COLS];
        for (int r = 0; r < rows; ++r)
            for (int c = 0; c < cols; ++c) acc[r][c] = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float* brow = bf + (size_t)k * N + j0;
            for (int r = 0; r < rows; ++r) {
                const float a = af[(size_t)(i0 + r) * K + k];
                for (int c = 0; c < cols; ++c) acc[r][c] = fmaf(a, brow[c], acc[r][c]);
            }
        }
        /* Zero padding up to a multiple of 16: fmaf(0, 0, acc) == acc for
         * acc != -0, and acc can never be -0 from a +0 start under RNE, so
         * the padded steps leave every accumulator unchanged. */
        (void)k_padded;
        for (int r = 0; r < rows; ++r)
            for (int c = 0; c < cols; ++c)
                C[(size_t)(i0 + r) * N + j0 + c] = kmcts_oracle_float_to_bf16(acc[r][c]);
    }
    free(af);
    free(bf);
    return 0;
}

/* ---------------------------------------------------------------- checks */

/* The reference harness's acceptance test.  out[0] = maximum_error,
 * out[1] = mean_error.  Returns 1 if every element passes, else 0. */
int kmcts_oracle_check(const uint16_t* C, const uint16_t* reference, size_t count,
                       double rtol, double atol, double* out) {
    double maximum_error = 0.0, error_sum = 0.0;
    int success = 1;
    for (size_t i = 0; i < count; ++i) {
        const double actual = kmcts_oracle_bf16_to_float(C[i]);
        const double expected = kmcts_oracle_bf16_to_float(reference[i]);
        const double error = fabs(actual - expected);
        if (error > maximum_error) maximum_error = error;
        error_sum += error;
        if (!isfinite(actual) || error > atol + rtol * fabs(expected)) success = 0;
    }
    out[0] = maximum_error;
    out[1] = count ? error_sum / (double)count : 0.0;
    return success;
}

/* Distance in BF16 units in the last place between two BF16 values, on the
 * monotone integer line (so +0 and -0 are 0 apart).  NaN yields 65535. */
static int32_t ordered(uint16_t v) {
    return (v & 0x8000u) ? -(int32_t)(v & 0x7fffu) : (int32_t)v;
}

uint32_t kmcts_oracle_ulp_distance(uint16_t a, uint16_t b) {
    if (((a & 0x7f80u) == 0x7f80u && (a & 0x7fu)) || ((b & 0x7f80u) == 0x7f80u && (b & 0x7fu)))
        return 65535u;
    int32_t d = ordered(a) - ordered(b);
    return (uint32_t)(d < 0 ? -d : d);
}

/* Histogram of ulp distances: hist[0..3] = count at 0, 1, 2, >2.
 * Returns the maximum distance. */
uint32_t kmcts_oracle_ulp_histogram(const uint16_t* C, const uint16_t* reference, size_t count,
                                    uint64_t* hist) {
    uint32_t worst = 0;
    hist[0] = hist[1] = hist[2] = hist[3] = 0;
    for (size_t i = 0; i < count; ++i) {
        uint32_t d = kmcts_oracle_ulp_distance(C[i], reference[i]);
        if (d > worst) worst = d;
        hist[d > 2 ? 3 : d] += 1;
    }
    return worst;
}
