/* CPU oracle for the NVFP4 activation quantiser, in C.  TEST INFRASTRUCTURE ONLY.
 *
 * A line-for-line arithmetic restatement of the reference's numpy quantiser (scripts/nvfp4_ref.py:43-82), used
 * by the tests to check the CUDA kernels bit-exactly at full size, and by bench.py's CPU-baseline leg.  It is
 * checked against tests/golden/ (which the reference's own functions produced) and against nvfp4_oracle.py in
 * tests/test_oracle_c.py.  Nothing on the product path links it.
 *
 * All block arithmetic is IEEE float64 in the same order as the reference:
 *   stored  = e4m3_round_pos(gscale * (bamax / 6.0))        scripts/nvfp4_ref.py:75-77
 *   local   = stored > 0 ? stored / gscale : 1.0             scripts/nvfp4_ref.py:78
 *   code    = e2m1_round(x / local)                          scripts/nvfp4_ref.py:79
 * Rounding: nearest, ties toward the smaller magnitude; e4m3 zero -> byte 0x80 (scripts/nvfp4_ref.py:47-50,57).
 * Build with -ffp-contract=off so no multiply-add is fused.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static double g_grid[127];      /* distinct finite non-negative e4m3 values, ascending */
static uint8_t g_grid_byte[127];
static int g_ready = 0;

static double e4m3_value(int b) {
    int e = (b >> 3) & 0xF, m = b & 7;
    double v = (e == 0) ? (m / 8.0) * ldexp(1.0, -6) : (1.0 + m / 8.0) * ldexp(1.0, e - 7);
    return (b & 0x80) ? -v : v;
}

static void init_tables(void) {
    if (g_ready) return;
    /* value 0 -> byte 0x80 (reference quirk: its value->byte dict lets -0.0 overwrite +0.0) */
    g_grid[0] = 0.0;
    g_grid_byte[0] = 0x80;
    for (int b = 1; b <= 0x7E; ++b) { g_grid[b] = e4m3_value(b); g_grid_byte[b] = (uint8_t)b; }
    g_ready = 1;
}

/* numpy.searchsorted(grid, x, side='left') for a sorted array of n values */
static int search_left(const double* grid, int n, double x) {
    int lo = 0, hi = n;
    while (lo < hi) { int mid = (lo + hi) >> 1; if (grid[mid] < x) lo = mid + 1; else hi = mid; }
    return lo;
}

/* scripts/nvfp4_ref.py:43-52 */
static void e4m3_round_pos(double x, uint8_t* byte, double* val) {
    int hi = search_left(g_grid, 127, x);
    if (hi > 126) hi = 126;
    int lo = hi - 1 < 0 ? 0 : hi - 1;
    int take_lo = fabs(x - g_grid[lo]) <= fabs(x - g_grid[hi]);
    int idx = take_lo ? lo : hi;
    *byte = g_grid_byte[idx];
    *val = g_grid[idx];
}

static const double k_mag[8] = {0, 0.5, 1, 1.5, 2, 3, 4, 6};

/* scripts/nvfp4_ref.py:54-61 */
static uint8_t e2m1_round(double x) {
    double a = fabs(x);
    int hi = search_left(k_mag, 8, a);
    if (hi > 7) hi = 7;
    int lo = hi - 1 < 0 ? 0 : hi - 1;
    int take_lo = fabs(a - k_mag[lo]) <= fabs(a - k_mag[hi]);
    uint8_t code = (uint8_t)(take_lo ? lo : hi);
    return code | (uint8_t)((x < 0) << 3);
}

static inline double bf16_to_double(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return (double)f;
}

static void quant_block(const double* xb, double g, uint8_t* packed8, uint8_t* sf) {
    double bamax = 0.0;
    for (int i = 0; i < 16; ++i) { double a = fabs(xb[i]); if (a > bamax) bamax = a; }
    double stored;
    e4m3_round_pos(g * (bamax / 6.0), sf, &stored);
    double local = stored > 0 ? stored / g : 1.0;
    for (int i = 0; i < 8; ++i) {
        uint8_t lo = e2m1_round(xb[2 * i] / local);
        uint8_t hi = e2m1_round(xb[2 * i + 1] / local);
        packed8[i] = (uint8_t)(lo | (hi << 4));
    }
}

/* Quantise bf16 rows: x [M,K] (bf16 bit patterns), packed [M,K/2], sf_logical [M,K/16]. */
void orc_quantize_rows_bf16(const uint16_t* x, int M, int K, float gscale, uint8_t* packed, uint8_t* sf_logical) {
    init_tables();
    const int kb = K / 16;
    const double g = (double)gscale;
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        double xb[16];
        for (int b = 0; b < kb; ++b) {
            const uint16_t* src = x + (size_t)m * K + (size_t)b * 16;
            for (int i = 0; i < 16; ++i) xb[i] = bf16_to_double(src[i]);
            quant_block(xb, g, packed + (size_t)m * (K / 2) + (size_t)b * 8, sf_logical + (size_t)m * kb + b);
        }
    }
}

/* Quantise fp32 rows (the legacy entry point's input type). */
void orc_quantize_rows_f32(const float* x, int M, int K, float gscale, uint8_t* packed, uint8_t* sf_logical) {
    init_tables();
    const int kb = K / 16;
    const double g = (double)gscale;
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        double xb[16];
        for (int b = 0; b < kb; ++b) {
            const float* src = x + (size_t)m * K + (size_t)b * 16;
            for (int i = 0; i < 16; ++i) xb[i] = (double)src[i];
            quant_block(xb, g, packed + (size_t)m * (K / 2) + (size_t)b * 8, sf_logical + (size_t)m * kb + b);
        }
    }
}

/* max |x| over n bf16 values, as float. */
float orc_amax_bf16(const uint16_t* x, long long n) {
    uint16_t best = 0;
#pragma omp parallel
    {
        uint16_t loc = 0;
#pragma omp for schedule(static) nowait
        for (long long i = 0; i < n; ++i) { uint16_t a = x[i] & 0x7FFF; if (a > loc) loc = a; }
#pragma omp critical
        { if (loc > best) best = loc; }
    }
    return (float)bf16_to_double(best);
}

/* logical [outer, K/16] -> 128x4 tiles, padding zero.  kernels/fp4_gemm.cu:21-33 */
void orc_swizzle_scales(const uint8_t* logical, uint8_t* swz, int outer, int K) {
    const int kb = K / 16, tile_cols = (kb + 3) / 4;
    const size_t total = (size_t)((outer + 127) / 128) * tile_cols * 512;
    memset(swz, 0, total);
    for (int m = 0; m < outer; ++m)
        for (int b = 0; b < kb; ++b) {
            size_t tile = (size_t)(m / 128) * tile_cols + (size_t)(b / 4);
            swz[tile * 512 + (m % 32) * 16 + ((m % 128) / 32) * 4 + (b % 4)] = logical[(size_t)m * kb + b];
        }
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Dequantise NVFP4 rows in float64: out[r, k] = e2m1(code) * (e4m3(scale) / gscale), the value order of
 * nvfp4_oracle.dequantize (scripts/ref_forward.py:51-64, dequant_linear).  packed [rows, K/2] (even element in the
 * low nibble), sf_logical [rows, K/16]. */
void orc_dequantize_rows(const uint8_t* packed, const uint8_t* sf_logical, int rows, int K, float gscale,
                         double* out) {
    static const double k_e2m1[16] = {0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6};
    const double g = (double)gscale;
    const int kb = K / 16;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t* pr = packed + (size_t)r * (K / 2);
        const uint8_t* sr = sf_logical + (size_t)r * kb;
        double* orow = out + (size_t)r * K;
        for (int b = 0; b < kb; ++b) {
            const double s = e4m3_value(sr[b]) / g;
            for (int i = 0; i < 8; ++i) {
                const uint8_t v = pr[b * 8 + i];
                orow[b * 16 + 2 * i] = k_e2m1[v & 15] * s;
                orow[b * 16 + 2 * i + 1] = k_e2m1[v >> 4] * s;
            }
        }
    }
}
