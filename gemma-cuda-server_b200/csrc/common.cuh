// common.cuh -- shared device/host helpers for the sm_100a NVFP4 library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nvfp4_b200.h"

namespace nvfp4b {

// ------------------------------------------------------------------------------------------------------------
// Host-side helpers
// ------------------------------------------------------------------------------------------------------------

// Records the failing cudaError_t for nvfp4b_last_cuda_error() and maps it to NVFP4B_ERR_CUDA.
int record_cuda_error(cudaError_t e);

// Status of the launch that was just issued (cudaGetLastError), as an NVFP4B status.
inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NVFP4B_OK : record_cuda_error(e);
}

// Streaming-multiprocessor count of the current device (cached per device).
int sm_count();

// Device address of the library's error word on the current device (cached per device; NULL on failure).
int* device_error_ptr();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch with cudaLaunchKernelEx (arguments converted to the kernel's own parameter types); returns the launch's
// NVFP4B status.  (Programmatic dependent launch was tried for the MoE layer's chain of kernels and measured slower:
// 137-140 vs 132 us per decode-size layer, whether the next kernel was released at the start or at the end of each
// block's work.)
template <typename... KArgs, typename... Args>
inline int launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                    Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    return e == cudaSuccess ? NVFP4B_OK : record_cuda_error(e);
}

inline size_t scale_bytes(int outer, int K) {
    const size_t tiles_r = (size_t)((outer + 127) / 128), tiles_c = (size_t)((K / 16 + 3) / 4);
    return tiles_r * tiles_c * 512;
}

constexpr float kGscaleNum = 2688.0f;   // 448 (e4m3 max) * 6 (e2m1 max)

// ------------------------------------------------------------------------------------------------------------
// NVFP4 numerics shared by the quantiser, the fused MoE dispatch and the GEMM epilogues.
//
// The target is the reference's numpy quantiser (scripts/nvfp4_ref.py:43-82), bit for bit:
//   t      = fl64(g * fl64(bamax / 6))                 e4m3 input, float64
//   stored = nearest e4m3 >= 0 to t, ties to the smaller value, 0 -> byte 0x80, > 448 -> 448
//   L      = stored > 0 ? fl64(stored / g) : 1
//   code   = #{ mid in {.25,.75,1.25,1.75,2.5,3.5,5} : mid < fl64(|x| / L) } | (x < 0 ? 8 : 0)
// The last line is the reference's "nearest e2m1, ties toward the smaller magnitude": every subtraction in its
// tie test is exact (Sterbenz), so the test reduces to comparing the float64 quotient with the midpoints.
//
// Per element the kernels evaluate the quotient in fp32 twice, scaled by (1 - 2^-20) and (1 + 2^-20); the fp32
// estimate is within 2^-22.9 relative of the float64 quotient, so the float64 quotient lies strictly between the
// two.  When both round (cvt.rn.satfinite.e2m1x2) to the same code no midpoint lies between them and that code is
// the reference's; when they differ, the element is recomputed exactly in float64.  The slow path is taken only
// for elements within ~1e-6 relative of a rounding boundary.
// ------------------------------------------------------------------------------------------------------------

__device__ __forceinline__ float gscale_from_amax(float amax) {
    return __fdiv_rn(kGscaleNum, fmaxf(amax, 1e-9f));
}

// 2^e as a double, e in the normal range.
__device__ __forceinline__ double pow2d(int e) {
    return __longlong_as_double((long long)(e + 1023) << 52);
}

// Nearest finite non-negative e4m3 value to t >= 0, ties toward the smaller value.  Returns the byte (0x80 for
// zero) and writes the value.
__device__ __forceinline__ uint32_t e4m3_encode_ties_low(double t, double* val) {
    if (!(t > 0.0)) { *val = 0.0; return 0x80u; }
    if (t >= 448.0) { *val = 448.0; return 0x7Eu; }
    int e = ilogb(t);
    const int es = e < -6 ? -6 : e;                 // values below 2^-6 share the subnormal step 2^-9
    const double step = pow2d(es - 3);
    const double n = floor(__dmul_rn(t, pow2d(3 - es)));
    const double lo = __dmul_rn(n, step), hi = __dmul_rn(n + 1.0, step);
    double v;
    if (lo == t) v = t;
    else v = (__dsub_rn(t, lo) <= __dsub_rn(hi, t)) ? lo : hi;
    *val = v;
    if (v == 0.0) return 0x80u;
    if (v < 0.015625) return (uint32_t)__dmul_rn(v, 512.0);             // subnormal: m * 2^-9
    const int E = ilogb(v);
    const uint32_t m = (uint32_t)__dmul_rn(__dsub_rn(__dmul_rn(v, pow2d(-E)), 1.0), 8.0);
    return ((uint32_t)(E + 7) << 3) | m;
}

// e4m3 byte -> float (0x80 and 0x00 decode to zero; NaN bytes are never produced here).
__host__ __device__ __forceinline__ float e4m3_to_float(uint32_t b) {
    const uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
    float mag;
    if (e == 0) {
        mag = (float)m * (1.0f / 512.0f);
    } else {
        union { uint32_t u; float f; } p;
        p.u = (e - 7u + 127u) << 23;
        mag = (1.0f + (float)m * 0.125f) * p.f;
    }
    return (b & 0x80u) ? -mag : mag;
}

struct BlockParams {
    uint32_t sf;    // stored e4m3 byte
    float invL;     // fp32 estimate of 1/L = g / stored (fast path)
    float stored;   // e4m3 value of the stored scale (exact in fp32; 0 for byte 0x80)
    float g;        // global scale
};

// Two fp32 -> e4m3 conversions, RNE with saturation to 448: lo goes to the low byte.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float hi, float lo) {
    uint16_t out;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(hi), "f"(lo));
    return out;
}

// Exact float64 block scale (the slow path, taken when the fp32 estimate is within 2^-20 of an e4m3 rounding
// boundary).
static __device__ __noinline__ uint32_t e4m3_scale_exact(float bamax, float g) {
    double stored;
    const double t = __dmul_rn((double)g, __ddiv_rn((double)bamax, 6.0));
    return e4m3_encode_ties_low(t, &stored);
}

// Block scale.  t = g * bamax / 6 is estimated in fp32 (within 3 * 2^-24 relative of the reference's float64
// value, or flushed to zero when far below the smallest e4m3 step); the estimate is scaled by (1 -/+ 2^-20) and
// both are rounded by the hardware (RNE, saturating).  Equal results mean no e4m3 rounding boundary lies between
// them, so that value is also the reference's ties-to-smaller rounding of the float64 t.
__device__ __forceinline__ BlockParams block_params(float bamax, float g) {
    BlockParams p;
    const float t = __fmul_rn(__fmul_rn(g, bamax), 0.16666667163372039795f);
    const uint32_t two = cvt_e4m3x2(__fmul_rn(t, 1.00000095367431640625f), __fmul_rn(t, 0.99999904632568359375f));
    uint32_t b = two & 0xFFu;
    if (__builtin_expect(b != (two >> 8), 0)) b = e4m3_scale_exact(bamax, g);
    if (b == 0u) b = 0x80u;                       // a zero scale is stored as 0x80 (reference quirk)
    p.sf = b;
    p.g = g;
    p.stored = e4m3_to_float(b & 0x7Fu);
    p.invL = (b & 0x7Fu) ? __fmul_rn(g, __frcp_rn(p.stored)) : 1.0f;
    return p;
}

// Exact float64 e2m1 code of x / L (the slow path); L = stored / g, or 1 for a zero scale.
static __device__ __noinline__ uint32_t e2m1_code_exact(float x, float stored, float g) {
    const double L = stored > 0.0f ? __ddiv_rn((double)stored, (double)g) : 1.0;
    const double y = __ddiv_rn(fabs((double)x), L);
    const uint32_t c = (uint32_t)(y > 0.25) + (uint32_t)(y > 0.75) + (uint32_t)(y > 1.25) + (uint32_t)(y > 1.75) +
                       (uint32_t)(y > 2.5) + (uint32_t)(y > 3.5) + (uint32_t)(y > 5.0);
    return c | (x < 0.0f ? 8u : 0u);
}

// Four cvt.rn.satfinite.e2m1x2: 8 floats -> 8 codes in one word, element 0 in the lowest nibble.
__device__ __forceinline__ uint32_t cvt_e2m1x8(float a0, float a1, float a2, float a3,
                                               float a4, float a5, float a6, float a7) {
    uint32_t out;
    asm("{\n\t.reg .b8 q0, q1, q2, q3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q0, %2, %1;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q1, %4, %3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q2, %6, %5;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q3, %8, %7;\n\t"
        "mov.b32 %0, {q0, q1, q2, q3};\n\t}"
        : "=r"(out)
        : "f"(a0), "f"(a1), "f"(a2), "f"(a3), "f"(a4), "f"(a5), "f"(a6), "f"(a7));
    return out;
}

// Codes of 8 consecutive elements v[0..7] of a block with parameters p.
__device__ __forceinline__ uint32_t encode8(const float* v, const BlockParams& p) {
    float lo[8], hi[8];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        // v * invL + 0: the +0 addend turns -0.0 into +0.0 (the reference gives code 0 for -0.0) while a
        // non-zero negative product keeps its sign even when it underflows.
        const float2 q = __ffma2_rn(make_float2(v[i], v[i + 1]), make_float2(p.invL, p.invL), make_float2(0.f, 0.f));
        const float2 l = __fmul2_rn(q, make_float2(0.99999904632568359375f, 0.99999904632568359375f));
        const float2 h = __fmul2_rn(q, make_float2(1.00000095367431640625f, 1.00000095367431640625f));
        lo[i] = l.x; lo[i + 1] = l.y;
        hi[i] = h.x; hi[i + 1] = h.y;
    }
    const uint32_t wl = cvt_e2m1x8(lo[0], lo[1], lo[2], lo[3], lo[4], lo[5], lo[6], lo[7]);
    uint32_t wh = cvt_e2m1x8(hi[0], hi[1], hi[2], hi[3], hi[4], hi[5], hi[6], hi[7]);
    uint32_t diff = wl ^ wh;
    if (__builtin_expect(diff != 0u, 0)) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if ((diff >> (4 * i)) & 0xFu) {
                const uint32_t c = e2m1_code_exact(v[i], p.stored, p.g);
                wh = (wh & ~(0xFu << (4 * i))) | (c << (4 * i));
            }
        }
    }
    return wh;
}

// Quantise one 16-element block: returns the scale byte, writes the 8 code bytes as two words.
__device__ __forceinline__ uint32_t quantize16(const float* v, float g, uint32_t& w0, uint32_t& w1) {
    float bamax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) bamax = fmaxf(bamax, fabsf(v[i]));
    const BlockParams p = block_params(bamax, g);
    w0 = encode8(v, p);
    w1 = encode8(v + 8, p);
    return p.sf;
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Magnitude of an e2m1 code 0..7: 0, 0.5, 1, 1.5, 2, 3, 4, 6.
__device__ __forceinline__ float e2m1_magnitude(uint32_t mag) {
    if (mag < 2u) return 0.5f * (float)mag;
    return __int_as_float((int)(((mag >> 1) - 1u + 127u) << 23)) * (1.0f + 0.5f * (float)(mag & 1u));
}

// Code of one element whose two bracket estimates straddle an e2m1 rounding boundary: the bracket codes are
// magnitudes mh - 1 and mh, so the only question is which side of the boundary b between them the reference's
// float64 quotient y = |x| / (stored / g) falls.  |x| * g (a bf16 times an fp32) differs from b * stored (exact in
// fp32) by at least 2^-32 relative unless the two are equal, far more than float64 rounding can move y, so the
// exact sign of |x| * g - b * stored decides -- taken in fp32 as (p - b*stored) + fma(|x|, g, -p) with p = fl(|x|*g)
// (Sterbenz: the difference is exact, the sum has the exact sign).  Only an exact tie repeats the reference's
// float64 arithmetic, where the rounding of y decides (ties go to the smaller magnitude).
__device__ __forceinline__ uint32_t e2m1_resolve(float x, uint32_t code_hi, const BlockParams& p) {
    const uint32_t mh = code_hi & 7u, ml = mh - 1u;
    const float b = 0.5f * (e2m1_magnitude(ml) + e2m1_magnitude(mh));
    const float ax = fabsf(x);
    float d;
    if (p.stored > 0.0f) {
        const float pr = ax * p.g;
        d = (pr - b * p.stored) + fmaf(ax, p.g, -pr);
    } else {
        d = ax - b;                                   // zero scale: L = 1
    }
    uint32_t mag = d > 0.0f ? mh : ml;
    if (__builtin_expect(d == 0.0f && p.stored > 0.0f, 0)) {
        const double L = __ddiv_rn((double)p.stored, (double)p.g);
        mag = __ddiv_rn((double)ax, L) > (double)b ? mh : ml;
    }
    return mag | (code_hi & 8u);
}

// Replaces, in the code word `c` of 8 elements (4 words of bf16 pairs), every nibble flagged in `diff` by its
// exact code (e2m1_resolve).  The word is picked with compile-time compares so the inputs stay in registers.  With
// bf16 data and g = 2688/amax a few percent of blocks hold an element within 2^-20 of a rounding boundary.
__device__ __forceinline__ uint32_t resolve_codes(uint32_t c, uint32_t diff, uint32_t w0, uint32_t w1, uint32_t w2,
                                                  uint32_t w3, const BlockParams& p) {
    while (diff) {
        const int i = (__ffs(diff) - 1) >> 2;        // element 0..7 of this group
        diff &= ~(0xFu << (4 * i));
        const int j = i >> 1;
        uint32_t wi = w0;
        wi = j == 1 ? w1 : wi;
        wi = j == 2 ? w2 : wi;
        wi = j == 3 ? w3 : wi;
        const float x = (i & 1) ? bf16hi(wi) : bf16lo(wi);
        c = (c & ~(0xFu << (4 * i))) | (e2m1_resolve(x, (c >> (4 * i)) & 0xFu, p) << (4 * i));
    }
    return c;
}

__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Value of a positive e4m3 byte (b < 0x7F) by the hardware conversion e4m3 -> f16 (exact: every e4m3 value,
// subnormals included, is an f16) -> f32.  The byte is fed to both halves of the pair, so lane order is moot.
__device__ __forceinline__ float e4m3_value(uint32_t b) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((unsigned short)(b | (b << 8))));
    return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}

// Quantise one 16-element block given as 8 words of bf16 pairs (element 0 in the low half): returns the scale byte
// and the 8 code bytes (element 0 in the low nibble of c0).  Fast path: the two bracket estimates of every code are
// x * (g / stored) * (1 -/+ 2^-20), formed as one FFMA2 per pair and bracket with multipliers folded per block
// (g / stored from rcp.approx: with the products it stays within 2^-22 of the exact quotient, well inside the
// 2^-20 bracket).  Equal codes from both brackets are the reference's codes; a block with any element whose
// brackets differ is finished by the float64 path for those elements only.
__device__ __forceinline__ uint32_t quantize16_bf16(const uint32_t (&w)[8], float g, uint32_t& c0, uint32_t& c1) {
    float f[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        f[2 * i] = bf16lo(w[i]);
        f[2 * i + 1] = bf16hi(w[i]);
    }
    float bamax = fabsf(f[0]);
#pragma unroll
    for (int i = 1; i < 16; ++i) bamax = fmaxf(bamax, fabsf(f[i]));
    const float t = __fmul_rn(__fmul_rn(g, bamax), 0.16666667163372039795f);
    const uint32_t two = cvt_e4m3x2(__fmul_rn(t, 1.00000095367431640625f), __fmul_rn(t, 0.99999904632568359375f));
    uint32_t b = two & 0xFFu;
    if (__builtin_expect(b != (two >> 8), 0)) b = e4m3_scale_exact(bamax, g);
    if (b == 0u) b = 0x80u;                       // a zero scale is stored as 0x80 (reference quirk)
    BlockParams p;
    p.sf = b;
    p.g = g;
    p.stored = (b & 0x7Fu) ? e4m3_value(b & 0x7Fu) : 0.0f;
    const float invL = (b & 0x7Fu) ? __fmul_rn(g, rcp_approx(p.stored)) : 1.0f;
    p.invL = invL;
    const float2 ml = make_float2(invL * 0.99999904632568359375f, invL * 0.99999904632568359375f);
    const float2 mh = make_float2(invL * 1.00000095367431640625f, invL * 1.00000095367431640625f);
    float lo[16], hi[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        // + 0: turns -0.0 into +0.0 (the reference gives code 0 for -0.0); a negative product keeps its sign.
        const float2 x2 = make_float2(f[2 * i], f[2 * i + 1]);
        const float2 l = __ffma2_rn(x2, ml, make_float2(0.f, 0.f));
        const float2 h = __ffma2_rn(x2, mh, make_float2(0.f, 0.f));
        lo[2 * i] = l.x; lo[2 * i + 1] = l.y;
        hi[2 * i] = h.x; hi[2 * i + 1] = h.y;
    }
    const uint32_t l0 = cvt_e2m1x8(lo[0], lo[1], lo[2], lo[3], lo[4], lo[5], lo[6], lo[7]);
    const uint32_t l1 = cvt_e2m1x8(lo[8], lo[9], lo[10], lo[11], lo[12], lo[13], lo[14], lo[15]);
    c0 = cvt_e2m1x8(hi[0], hi[1], hi[2], hi[3], hi[4], hi[5], hi[6], hi[7]);
    c1 = cvt_e2m1x8(hi[8], hi[9], hi[10], hi[11], hi[12], hi[13], hi[14], hi[15]);
    if (__builtin_expect(((l0 ^ c0) | (l1 ^ c1)) != 0u, 0)) {
        c0 = resolve_codes(c0, l0 ^ c0, w[0], w[1], w[2], w[3], p);
        c1 = resolve_codes(c1, l1 ^ c1, w[4], w[5], w[6], w[7], p);
    }
    return b;
}

// The straight-line part of quantize16_bf16: the block scale and codes from the fp32 brackets only, no exact paths.
// Returns the scale byte, with bit 8 set when the result is not proven to be the reference's (the two block-scale
// brackets or the two code brackets of some element disagree); such a block must be redone by quantize16_bf16.
__device__ __forceinline__ uint32_t quantize16_bf16_fast(const uint32_t (&w)[8], float g, uint32_t& c0,
                                                         uint32_t& c1) {
    float f[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        f[2 * i] = bf16lo(w[i]);
        f[2 * i + 1] = bf16hi(w[i]);
    }
    float bamax = fabsf(f[0]);
#pragma unroll
    for (int i = 1; i < 16; ++i) bamax = fmaxf(bamax, fabsf(f[i]));
    const float t = __fmul_rn(__fmul_rn(g, bamax), 0.16666667163372039795f);
    const uint32_t two = cvt_e4m3x2(__fmul_rn(t, 1.00000095367431640625f), __fmul_rn(t, 0.99999904632568359375f));
    uint32_t b = two & 0xFFu;
    const uint32_t flag = b != (two >> 8) ? 0x100u : 0u;
    if (b == 0u) b = 0x80u;                       // a zero scale is stored as 0x80 (reference quirk)
    const float stored = (b & 0x7Fu) ? e4m3_value(b & 0x7Fu) : 0.0f;
    const float invL = (b & 0x7Fu) ? __fmul_rn(g, rcp_approx(stored)) : 1.0f;
    const float2 ml = make_float2(invL * 0.99999904632568359375f, invL * 0.99999904632568359375f);
    const float2 mh = make_float2(invL * 1.00000095367431640625f, invL * 1.00000095367431640625f);
    float lo[16], hi[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float2 x2 = make_float2(f[2 * i], f[2 * i + 1]);
        const float2 l = __ffma2_rn(x2, ml, make_float2(0.f, 0.f));
        const float2 h = __ffma2_rn(x2, mh, make_float2(0.f, 0.f));
        lo[2 * i] = l.x; lo[2 * i + 1] = l.y;
        hi[2 * i] = h.x; hi[2 * i + 1] = h.y;
    }
    const uint32_t l0 = cvt_e2m1x8(lo[0], lo[1], lo[2], lo[3], lo[4], lo[5], lo[6], lo[7]);
    const uint32_t l1 = cvt_e2m1x8(lo[8], lo[9], lo[10], lo[11], lo[12], lo[13], lo[14], lo[15]);
    c0 = cvt_e2m1x8(hi[0], hi[1], hi[2], hi[3], hi[4], hi[5], hi[6], hi[7]);
    c1 = cvt_e2m1x8(hi[8], hi[9], hi[10], hi[11], hi[12], hi[13], hi[14], hi[15]);
    return b | flag | ((((l0 ^ c0) | (l1 ^ c1)) != 0u) ? 0x100u : 0u);
}

}  // namespace nvfp4b
