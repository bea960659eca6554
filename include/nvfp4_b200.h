/* nvfp4_b200.h -- C ABI of the B200 (sm_100a) NVFP4 quantised-matmul library (libnvfp4_b200.so).
 *
 * Plain pointers, sizes and an opaque stream handle (a cudaStream_t passed as void*; NULL = the legacy default
 * stream).  Every function that launches work returns an int status: 0 on success, a negative NVFP4B_ERR_* code
 * otherwise.  No function allocates device memory, synchronises the host, or calls a CUDA API that is illegal
 * during stream capture, unless its comment says so.  All device buffers are owned by the caller.
 *
 * NVFP4 conventions shared by every entry point:
 *   codes   : e2m1, two per byte, the even-index element in the low nibble                   [rows, K/2] uint8
 *   scales  : one e4m3 byte per 16-element block along K, stored in the 128x4-tile layout the tensor cores read
 *             (tile = 128 rows x 4 blocks = 512 bytes, tiles row-major; within a tile the byte of (m, b) is at
 *             (m%32)*16 + ((m%128)/32)*4 + (b%4)); rows padded to 128 and blocks to 4 with zero bytes.
 *             Size: nvfp4b_scale_buffer_bytes(rows, K).
 *   gscale  : fp32 per-tensor global scale in the compressed-tensors convention, 2688 / amax.  Dequantised value
 *             = e2m1(code) * e4m3(scale) / gscale.
 * Rounding follows the reference's numpy quantiser (scripts/nvfp4_ref.py:43-82) bit for bit: float64 block
 * arithmetic, nearest with ties toward the smaller magnitude for both e4m3 and e2m1, an all-zero block stores
 * scale byte 0x80.
 */
#ifndef NVFP4_B200_H
#define NVFP4_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum nvfp4b_status {
    NVFP4B_OK = 0,
    NVFP4B_ERR_SHAPE = -1,   /* a dimension is out of range or not a multiple the path requires */
    NVFP4B_ERR_ALIGN = -2,   /* a pointer or row pitch is not 16-byte aligned */
    NVFP4B_ERR_NULL = -3,    /* a required pointer is NULL */
    NVFP4B_ERR_CUDA = -4,    /* a CUDA call failed; nvfp4b_last_cuda_error() has the cudaError_t */
    NVFP4B_ERR_ARCH = -5,    /* the current device is not an sm_100 part */
    NVFP4B_ERR_TIMEOUT = -6, /* a bounded device-side wait expired (no fault, the context stays usable) */
    NVFP4B_ERR_ARG = -7,     /* an enum/flag argument has an unknown value */
    NVFP4B_ERR_SCRATCH = -8  /* the problem needs more scratch than a fixed-size (no-allocation) entry point holds */
};

/* Library version string. */
const char* nvfp4b_version(void);
/* cudaError_t of the most recent failing CUDA call made by this thread inside the library (0 if none). */
int nvfp4b_last_cuda_error(void);

/* Bytes of a swizzled scale buffer for a [outer, K] NVFP4 operand.  Same value as the reference's
 * nvfp4_scale_buffer_bytes (kernels/fp4_gemm.cu:14-19). */
size_t nvfp4b_scale_buffer_bytes(int outer, int K);

/* ---- activation quantiser (replaces kernels/nvfp4_quant.cu:15-57; adds bf16 input and device amax) ---------- */

/* d_amax[0] = max |x| over n bf16 values (x is bf16 bit patterns, 16-byte aligned).  Zeroes d_amax first (an
 * async memset on the stream), then one reduction kernel. */
int nvfp4b_amax_bf16(const void* x, long long n, float* d_amax, void* stream);

/* Quantise x [M, K] (row-major, bf16 bit patterns) to NVFP4.  K % 16 == 0; x, packed and scales 16-byte aligned.
 * Global scale: if d_amax is NULL the host value `gscale` is used (static scale, the reference contract of
 * include/nvfp4_quant.h:10-11); otherwise gscale = 2688 / max(d_amax[0], 1e-9) is computed on the device as one
 * correctly rounded fp32 division (dynamic scale; pair with nvfp4b_amax_bf16 on the same stream).
 * packed [M, K/2]; scales: nvfp4b_scale_buffer_bytes(M, K) bytes, fully written including the zero padding. */
int nvfp4b_quantize_bf16(const void* x, int M, int K, float gscale, const float* d_amax,
                         uint8_t* packed, uint8_t* scales, void* stream);

/* Same as nvfp4b_quantize_bf16 for fp32 input (the reference entry point's input type). */
int nvfp4b_quantize_f32(const float* x, int M, int K, float gscale, const float* d_amax,
                        uint8_t* packed, uint8_t* scales, void* stream);

/* Device relayout of logical scales [outer, K/16] into the tile layout (padding zeroed).  Device-side twin of
 * the reference's host nvfp4_swizzle_scales (kernels/fp4_gemm.cu:21-33). */
int nvfp4b_swizzle_scales(const uint8_t* logical, uint8_t* swizzled, int outer, int K, void* stream);

/* ---- W4A4 NVFP4 GEMM (replaces the cuBLASLt call in kernels/fp4_gemm.cu:113-162) ----------------------------- */

enum nvfp4b_out_kind {
    NVFP4B_OUT_BF16_ROWMAJOR = 0, /* D[m*ldd + n] bf16 */
    NVFP4B_OUT_F32_COLMAJOR = 1,  /* D[m + n*ldd] fp32 (the reference nvfp4_gemm contract, ldd = M) */
    NVFP4B_OUT_F32_ROWMAJOR = 2   /* D[m*ldd + n] fp32 */
};

/* D = alpha * A @ B^T with A = activations [M, K] NVFP4 and B = weights [N, K] NVFP4 (both K-major codes plus
 * tile-layout scales), fp32 accumulation on the tensor cores (tcgen05 kind::mxf4nvf4, e4m3 scales per 16).
 * alpha = a_dequant * b_dequant where each dequant multiplier is 1/gscale; if d_a_amax is not NULL the activation
 * multiplier is instead 1 / (2688 / max(d_a_amax[0], 1e-9)) computed on the device (dynamic activation scale),
 * i.e. alpha = b_dequant / gscale(amax).  K % 32 == 0 (16-byte rows), pointers 16-byte aligned, ldd >= row length.
 * Any M, N >= 1. */
int nvfp4b_gemm(const uint8_t* a, const uint8_t* a_scales, float a_dequant, const float* d_a_amax,
                const uint8_t* b, const uint8_t* b_scales, float b_dequant,
                int M, int N, int K, void* d, int out_kind, long long ldd, void* stream);

/* Selects the dense GEMM tile configuration for subsequent calls in this process: 0 = automatic (default),
 * 1 = 128x256 tiles, 4-stage pipeline, one TMEM accumulator; 2 = 128x128 tiles, 6 stages, two accumulators;
 * 3 = 256x256 tiles computed by a CTA pair (cluster of two, tcgen05 cta_group::2), 5 stages. */
int nvfp4b_gemm_set_tile_config(int config);

/* Reads the library's device-side error word (set by a kernel whose bounded wait expired, see
 * NVFP4B_ERR_TIMEOUT) and optionally clears it.  Synchronous (cudaMemcpyFromSymbol): not for use during capture.
 * Returns 0 if no kernel reported an error. */
int nvfp4b_read_device_error(int reset);

/* Measurement (no counterpart in the reference): reads a [rows, row_bytes] byte matrix (row_bytes % 128 == 0,
 * 16-byte aligned) through the TMA path the GEMMs use -- boxes of 256 rows x 128 bytes into a 4-stage shared-memory
 * ring, one persistent CTA per SM -- and discards it.  bench.py times it at the byte count of a weight-stream-bound
 * kernel: the ceiling that kernel's stream can reach at its size. */
int nvfp4b_hbm_read_stream(const void* p, long long rows, int row_bytes, void* stream);

/* ---- W4A16 (replaces fp4_gemv / w4a16_gemm, kernels/fp4_gemm.cu:45-111) ----------------------------------- */

/* out[M, N] (fp32 row-major) = x16[M, K] (fp16 row-major) @ dequant(W[N, K])^T with raw, unswizzled weight codes
 * wp [N, K/2] and e4m3 scales ws [N, K/16]; dequant = code * e4m3 / w_gscale.  K % 16 == 0; any M (the
 * reference's kernel is limited to M <= 16); x16 2-byte aligned.  16-byte aligned operands with K % 32 == 0 take
 * the tensor-core paths (TMA-fed for M <= 2 with K % 256 == 0 and 16-byte aligned scales, register-fed for M <= 8,
 * passes of 16 rows for larger M with K % 64 == 0, each pass reading the weights once), anything else a
 * byte-granular one.  Sums are fp32 in every path. */
int nvfp4b_w4a16_gemm(float* out, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16,
                      int M, int N, int K, void* stream);

/* ---- Dense Linear (the call site of src/forward.cu:424-445, linear()) ----------------------------------------- */

/* d_amax[0] = max |x| over n fp32 values (16-byte aligned); zeroes d_amax first, then one reduction kernel. */
int nvfp4b_amax_f32(const float* x, long long n, float* d_amax, void* stream);

enum nvfp4b_linear_mode {
    NVFP4B_LINEAR_AUTO = 0,   /* W4A4 when M >= NVFP4B_LINEAR_W4A4_MIN_M (prefill), W4A16 otherwise (decode) */
    NVFP4B_LINEAR_W4A16 = 1,  /* fp16 activations x dequantised weights, fp32 accumulate (the reference's path) */
    NVFP4B_LINEAR_W4A4 = 2    /* activations quantised to NVFP4, tcgen05 NVFP4 GEMM */
};
#define NVFP4B_LINEAR_W4A4_MIN_M 128

/* Device bytes of the workspace nvfp4b_linear needs for an [M, K] input (caller allocates, 16-byte aligned). */
size_t nvfp4b_linear_workspace_bytes(int M, int K);

/* out[M, N] (fp32 row-major, ld N) = in[M, K] (fp32 row-major) @ W[N, K]^T with W in NVFP4: codes w [N, K/2],
 * dequant code * e4m3 / w_gscale.  The W4A16 path reads the raw scales w_scales [N, K/16] (as the reference's
 * Linear does); the W4A4 path reads the tile-layout copy w_scales_tiled (nvfp4b_scale_buffer_bytes(N, K), made
 * once at load, like Model::wscale in src/forward.cu:369-376) and quantises `in` with the activation global scale
 * a_gscale (static, compressed-tensors form 2688/amax), or, if a_gscale <= 0, with the dynamic scale of the
 * device amax of `in`.  Only the pointer the chosen path reads may be NULL otherwise.  The W4A4 path needs
 * K % 32 == 0.  Results: W4A4 = the oracle's float64 dequant-matmul of the quantised operands within fp32
 * accumulation error; W4A16 = the fp16 activations times the dequantised weights in fp32.  No allocation, no
 * synchronisation (capture-safe). */
int nvfp4b_linear(float* out, const float* in, int M, int N, int K, const uint8_t* w, const uint8_t* w_scales,
                  const uint8_t* w_scales_tiled, float w_gscale, float a_gscale, int mode, void* workspace,
                  size_t workspace_bytes, void* stream);

/* ---- MoE top-k grouped expert FFN (replaces the router and expert kernels of src/forward.cu:193-321 and the
 *      orchestration of moe(), src/forward.cu:516-553) ------------------------------------------------------------
 *
 * out[t] (+)= sum_j w[t,j] * W2_e (gelu_tanh(W1_e x_t) * (W3_e x_t)),  e = ids[t,j], j < topk
 * with x quantised to NVFP4 once per token (global scale of the layer input) and the intermediate h quantised to
 * NVFP4 in the gate/up epilogue with a static per-expert global scale (compressed-tensors "dynamic: local" block
 * scales + static global scale).  Expert weights live in one arena: */
typedef struct nvfp4b_moe_experts {
    int num_experts;            /* E */
    int hidden;                 /* H: model width, % 256 == 0 */
    int inter;                  /* I: expert intermediate width, % 32 == 0 */
    const uint8_t* w13;         /* [E, 2I, H/2] codes; rows of gate (W1) and up (W3) interleaved in groups of 16:
                                   row 32g + r = gate row 16g + r, row 32g + 16 + r = up row 16g + r (r < 16) */
    const uint8_t* w13_scales;  /* E consecutive tile-layout scale buffers of nvfp4b_scale_buffer_bytes(2I, H) */
    const uint8_t* w2;          /* [E, H, I/2] codes of the down projection (W2) */
    const uint8_t* w2_scales;   /* E consecutive scale buffers of nvfp4b_scale_buffer_bytes(H, I) */
    const float* w1_gscale;     /* [E] device: global scales of gate, up and down weights */
    const float* w3_gscale;
    const float* w2_gscale;
    const float* a2_gscale;     /* [E] device: static global scale of the down projection's input h */
} nvfp4b_moe_experts;

/* Device bytes of the workspace nvfp4b_moe_forward needs for T tokens (caller allocates, 256-byte aligned). */
size_t nvfp4b_moe_workspace_bytes(int T, int H, int I, int E, int topk);

/* Rows of the expert-sorted dispatch buffers (every expert segment padded to a multiple of 128 rows). */
int nvfp4b_moe_max_rows(int T, int E, int topk);

/* Router: logits = x @ proj^T on the tensor cores (bf16, fp32 accumulate, split along K), then per token softmax
 * over the E experts, top-k (ties to the lower expert id), renormalised to sum 1 and multiplied by
 * per_expert_scale[e] (if not NULL).  With norm != 0 the logits are scaled per token by H^-0.5 / rms(x) first
 * (the reference's rmsnorm-without-weight * scale * H^-0.5, with `scale` folded into proj by the caller).
 * x [T, H] bf16, proj [E, H] bf16; E % 32 == 0, E <= 256, topk <= 16.  ids [T, topk] int32, weights fp32. */
int nvfp4b_moe_route(const void* x, int T, int H, const void* proj, int E, int topk, const float* per_expert_scale,
                     int norm, int* ids, float* weights, void* workspace, void* stream);

/* nvfp4b_moe_route without a workspace argument; it allocates nothing.  No counterpart in the reference (whose router
 * kernels, src/forward.cu:192-234, write into model-owned buffers): it serves callers that cannot allocate or pass
 * scratch, e.g. a decode loop that reserves all of its memory up front.  The split-K partial logits live in a
 * fixed 4 MiB device array inside the library, one per device: T * E must be <= 262144 (T <= 2048 at E = 128), larger
 * calls return NVFP4B_ERR_SCRATCH.  Calls that overlap in time on one device race on that array: order them on one
 * stream.  The first call on each device looks the array up (and loads the library's module there); make it before
 * any stream capture that should contain this call.  Results equal nvfp4b_moe_route's. */
int nvfp4b_moe_route_noalloc(const void* x, int T, int H, const void* proj, int E, int topk,
                             const float* per_expert_scale, int norm, int* ids, float* weights, void* stream);

/* Whole MoE layer: dispatch (counting sort of the T*topk assignments by expert, stable in token order),
 * quantisation of x fused into the dispatch scatter, grouped gate/up GEMM with the gelu_tanh(gate)*up epilogue
 * requantised to NVFP4, grouped down GEMM whose epilogue scales each row by its router weight into an fp16 row
 * buffer, and a combine summing each token's topk rows in slot order in fp32 into out[t] (fp32 [T, H];
 * bit-reproducible).  flags: NVFP4B_MOE_* (ACCUMULATE adds onto out, e.g. the residual; ATOMIC uses fp32 atomic
 * adds instead).  ids/weights come from nvfp4b_moe_route or the caller.  Activation global scale: in_gscale, or
 * 2688 / max(*d_in_amax, 1e-9) on the device if d_in_amax is not NULL. */
enum nvfp4b_moe_flags {
    NVFP4B_MOE_ACCUMULATE = 1,  /* add the layer output onto out instead of overwriting it */
    NVFP4B_MOE_ATOMIC = 2       /* fp32 atomic adds into out instead of the (default, bit-reproducible) slot-ordered
                                   combine over an fp16 row buffer */
};
int nvfp4b_moe_forward(const void* x, int T, const int* ids, const float* weights, int topk,
                       const nvfp4b_moe_experts* experts, float in_gscale, const float* d_in_amax, float* out,
                       int flags, void* workspace, void* stream);

/* nvfp4b_moe_forward with the MoE input's RMSNorm fused into the quantise-dispatch (the reference normalises the
 * residual with pre_feedforward_layernorm_2 before its experts, src/forward.cu:535, kernels/elementwise.cu:10-22):
 * each token row is x * rsqrt(mean(x^2) + eps) * norm_weight in fp32 (norm_weight bf16 [H], 16-byte aligned) and
 * those fp32 values are quantised -- the normalised activations are never written.  Static activation global scale
 * only (in_gscale > 0, e.g. the checkpoint's input_global_scale): a dynamic one would need the normalised amax first. */
int nvfp4b_moe_forward_norm(const void* x, int T, const int* ids, const float* weights, int topk,
                            const nvfp4b_moe_experts* experts, const void* norm_weight, float eps, float in_gscale,
                            float* out, int flags, void* workspace, void* stream);

/* nvfp4b_moe_forward for a stack of layers on a residual stream: the combine also writes each finished out row
 * rounded to bf16 (RNE) into x_next [T, H] and max |x_next| into *d_amax_next (zeroed by this call after the layer
 * has read its own inputs, so x_next/d_amax_next may be the layer's own x/d_in_amax).  That is the next layer's
 * input and dynamic-scale amax, without a separate cast and amax pass.  NVFP4B_MOE_ATOMIC is not allowed here. */
int nvfp4b_moe_forward_chain(const void* x, int T, const int* ids, const float* weights, int topk,
                             const nvfp4b_moe_experts* experts, float in_gscale, const float* d_in_amax, float* out,
                             int flags, void* workspace, void* x_next, float* d_amax_next, void* stream);

/* The router fused into the MoE prologue: nvfp4b_moe_route followed by nvfp4b_moe_forward (x_next, d_amax_next
 * NULL) or nvfp4b_moe_forward_chain (both given), with the same results, in one call of seven kernel launches: the
 * router GEMM, the top-k with the dispatch's per-chunk ranking in the same kernel, the segment plan, the quantise-
 * scatter, the grouped gate/up and down GEMMs and the combine (the chained amax is reset inside the down GEMM, no
 * memset).  The router is over all experts->num_experts experts (proj [E, H] bf16; per_expert_scale and norm as for
 * nvfp4b_moe_route); ids [T, topk] int32 and weights [T, topk] fp32 receive the routing.  Replaces the reference's
 * k_router_hn/scores/top8 + moe() sequence (src/forward.cu:193-231, :516-553).  workspace:
 * nvfp4b_moe_workspace_bytes(T, H, I, E, topk). */
int nvfp4b_moe_layer(const void* x, int T, const void* proj, int topk, const float* per_expert_scale, int norm,
                     const nvfp4b_moe_experts* experts, float in_gscale, const float* d_in_amax, float* out,
                     int flags, int* ids, float* weights, void* workspace, void* x_next, float* d_amax_next,
                     void* stream);

/* The three stages of nvfp4b_moe_forward, callable one by one (same stream, same workspace, in this order):
 * dispatch (plan + quantise-scatter of x), gate/up grouped GEMM (writes the NVFP4 intermediate), down grouped GEMM
 * + weighted combine into out (flags as for nvfp4b_moe_forward). */
int nvfp4b_moe_dispatch(const void* x, int T, const int* ids, const float* weights, int topk,
                        const nvfp4b_moe_experts* experts, float in_gscale, const float* d_in_amax, void* workspace,
                        void* stream);
int nvfp4b_moe_gate_up(int T, int topk, const nvfp4b_moe_experts* experts, float in_gscale, const float* d_in_amax,
                       void* workspace, void* stream);
int nvfp4b_moe_down(int T, int topk, const float* weights, const nvfp4b_moe_experts* experts, float* out,
                    int flags, void* workspace, void* stream);

/* Calibration pass: runs dispatch and the gate/up GEMM and writes, per expert, max |h| over the rows routed to it
 * into h_amax[E] (device, fp32; zeroed first).  Static down-projection input scales are then 2688 / h_amax. */
int nvfp4b_moe_calibrate(const void* x, int T, const int* ids, const float* weights, int topk,
                         const nvfp4b_moe_experts* experts, float in_gscale, const float* d_in_amax, float* h_amax,
                         void* workspace, void* stream);

/* Debug/test view of the workspace after nvfp4b_moe_forward or _calibrate: device pointers to the dispatch plan
 * and the NVFP4 intermediate (see the field comments).  Pure pointer arithmetic, no CUDA call. */
typedef struct nvfp4b_moe_view {
    int* m_tiles;          /* [1] 128-row blocks in use */
    int* tile_expert;      /* [max_rows/128] expert of each row block */
    int* seg_start;        /* [E] first row of each expert segment */
    int* seg_count;        /* [E] real rows of each expert */
    int* row_token;        /* [max_rows] token of each row, -1 for padding */
    float* row_weight;     /* [max_rows] router weight of each row */
    int* row_assign;       /* [max_rows] assignment (token * topk + slot) of each row, -1 for padding */
    uint16_t* y;           /* [T*topk, H] fp16 (IEEE binary16) weighted expert outputs, assignment-major */
    int* dest;             /* [T*topk] row of each (token, slot) */
    uint8_t* a_codes;      /* [max_rows, H/2] quantised x, expert-sorted */
    uint8_t* a_scales;
    uint8_t* h_codes;      /* [max_rows, I/2] quantised h */
    uint8_t* h_scales;
} nvfp4b_moe_view;
int nvfp4b_moe_workspace_view(void* workspace, int T, int H, int I, int E, int topk, nvfp4b_moe_view* view);

/* Packs one expert's checkpoint tensors into the arena layout: gate/up codes [I, H/2] each and their logical
 * (unswizzled, [I, H/16]) e4m3 scales -> interleaved w13 rows + tile-layout scales; down codes are copied and its
 * logical scales [H, I/16] swizzled.  dst pointers address expert e's slots inside the arena.  Load-time only. */
int nvfp4b_moe_pack_expert(const uint8_t* gate, const uint8_t* gate_scales, const uint8_t* up,
                           const uint8_t* up_scales, const uint8_t* down, const uint8_t* down_scales, int H, int I,
                           uint8_t* w13_dst, uint8_t* w13_scales_dst, uint8_t* w2_dst, uint8_t* w2_scales_dst,
                           void* stream);

/* ---- expert parallelism: E experts sharded over G ranks, E/G consecutive experts per rank -------------------------
 *
 * One MoE layer on G ranks (the collectives are the caller's, e.g. NCCL all-to-all over NVLink).  Records travel in
 * fixed slots, `capacity` per (source, destination) pair, so no step needs the counts on the host (a layer can be
 * captured in a CUDA graph):
 *   source rank:  nvfp4b_moe_route -> nvfp4b_ep_dispatch (records [G][capacity], per-rank counts)
 *   collectives:  all-to-all of the counts (G ints) and of the record slots (capacity records per rank pair)
 *   expert rank:  nvfp4b_ep_expert_forward on the received slots (its E/G local experts)
 *   collectives:  all-to-all of the output row slots (fp16 [G * capacity, H], the workspace view's y) back
 *   source rank:  nvfp4b_ep_combine (slot-ordered sum into out; bit-identical to nvfp4b_moe_forward at G = 1).
 * A record carries the token's e2m1 codes, its logical e4m3 scales, the destination-local expert, the router weight
 * and the activation global scale the codes were made with (ranks quantise with their own dynamic scale).  A rank
 * pair with more than `capacity` records sets *overflow (the excess is dropped): capacity = T * topk can never
 * overflow; a smaller one trades all-to-all bytes for a check of the flag after the step. */

/* Bytes of one record: H/2 + H/16 + 16 (H % 256 == 0), 0 otherwise. */
size_t nvfp4b_ep_record_bytes(int H);

/* Source side: plans and packs the T*topk assignments (ids in [0, E), E % G == 0) into `records` (G * capacity
 * slots of nvfp4b_ep_record_bytes(H); destination d's records are slots [d * capacity, d * capacity + count)),
 * send_counts[G] (device int32) = per-destination counts (at most capacity), *overflow |= 1 if any pair exceeds
 * capacity.  workspace: nvfp4b_moe_workspace_bytes(T, H, 32, E, topk); keep it until nvfp4b_ep_combine. */
int nvfp4b_ep_dispatch(const void* x, int T, int H, const int* ids, const float* weights, int topk, int E, int G,
                       int capacity, float in_gscale, const float* d_in_amax, void* workspace, uint8_t* records,
                       int* send_counts, int* overflow, void* stream);

/* Expert side: the G * capacity received record slots (slot s * capacity + j is a record iff j < recv_counts[s],
 * recv_counts on the device) through the local experts (experts->num_experts = E/G): the weighted fp16 output row
 * of slot i is left at row i of the workspace's y.  workspace: nvfp4b_moe_workspace_bytes(G * capacity, H, I,
 * E/G, 1). */
int nvfp4b_ep_expert_forward(const uint8_t* records, int G, int capacity, const int* recv_counts,
                             const nvfp4b_moe_experts* experts, void* workspace, void* stream);

/* Source side: out[t] (+)= sum over slots j, in order, of y_back[record slot of (t, j)], fp32 accumulation;
 * y_back holds the returned row slots in this rank's record-slot order.  flags: NVFP4B_MOE_ACCUMULATE or 0. */
int nvfp4b_ep_combine(const uint16_t* y_back, int T, int H, int topk, int E, const void* workspace, float* out,
                      int flags, void* stream);

/* ---- Expert parallelism over NVLink peer memory (one process per GPU, no collective library on the data path) --
 *
 * The same layer with the two all-to-alls fused into the kernels around them: the source rank's pack kernel stores
 * each record straight into the destination rank's receive slots (its block `rank`), and the expert rank's down-
 * projection epilogue stores each weighted fp16 row straight into the source rank's return rows (block `rank`),
 * both with plain stores to peer memory over NVLink.  Only the records that exist cross the link.  Completion is
 * published per (rank pair, layer) with a release store of the layer's epoch to a flag word in the receiver's
 * memory, written by the last block of the producing kernel after a system-scope fence; the receiving kernels
 * (record scatter, combine) acquire it with a bounded spin (NVFP4B_ERR_TIMEOUT in the device error word after
 * ~10 s; the kernel then goes on and the context stays usable).  Layer order per rank, all on one stream:
 *   nvfp4b_ep_p2p_dispatch -> nvfp4b_ep_p2p_expert_forward -> nvfp4b_ep_p2p_combine
 * Results are bit-identical to nvfp4b_moe_forward over all experts (same quantisation, same slot-ordered sum).
 * Exchange buffers live in one device allocation per rank (nvfp4b_ipc_alloc), shared with the other ranks through
 * CUDA IPC handles; every pointer below is a device pointer in the calling rank's address space. */
typedef struct nvfp4b_ep_peers {
    int rank, G, capacity;        /* this rank, ranks, record slots per (source, destination) pair */
    uint8_t* const* recv;         /* device array [G]: rank g's receive slots [G * capacity] records */
    uint16_t* const* back;        /* device array [G]: rank g's return rows [G * capacity, H] fp16 */
    int* const* counts;           /* device array [G]: rank g's receive counts [G] int32 */
    unsigned* const* flags;       /* device array [G]: rank g's flag words [2G] (records landed / rows landed) */
    uint8_t* my_recv;             /* this rank's own buffers: entries `rank` of the arrays above */
    uint16_t* my_back;
    int* my_counts;
    unsigned* my_flags;
    unsigned* state;              /* this rank's 4 private words (layer epoch, completion counters) */
} nvfp4b_ep_peers;

/* Bytes of one rank's exchange buffers and their offsets inside it (each 256-byte aligned): receive slots, return
 * rows, counts, flags, state.  offsets[5] may be NULL.  The flags, counts and state must be zero before the first
 * layer (nvfp4b_ipc_alloc zeroes the whole allocation). */
size_t nvfp4b_ep_p2p_buffer_bytes(int G, int capacity, int H, size_t* offsets);

/* Source side: as nvfp4b_ep_dispatch, records stored into the destinations' receive slots and counts, then the
 * records-landed flags raised and this rank's layer epoch advanced.  *overflow |= 1 if a destination would get
 * more than capacity records (excess not sent).  workspace: nvfp4b_moe_workspace_bytes(T, H, 32, E, topk), kept
 * until nvfp4b_ep_p2p_combine. */
int nvfp4b_ep_p2p_dispatch(const void* x, int T, int H, const int* ids, const float* weights, int topk, int E,
                           float in_gscale, const float* d_in_amax, void* workspace, const nvfp4b_ep_peers* peers,
                           int* overflow, void* stream);

/* Expert side: waits for every source's records of this layer, runs the local experts (experts->num_experts =
 * E / G) and stores the weighted rows into the sources' return rows, then raises the rows-landed flags.
 * workspace: nvfp4b_moe_workspace_bytes(G * capacity, H, I, E / G, 1). */
int nvfp4b_ep_p2p_expert_forward(const nvfp4b_moe_experts* experts, void* workspace, const nvfp4b_ep_peers* peers,
                                 void* stream);

/* Source side: waits for every expert rank's rows of this layer and sums them into out in slot order (flags:
 * NVFP4B_MOE_ACCUMULATE or 0).  `workspace` is the one given to nvfp4b_ep_p2p_dispatch. */
int nvfp4b_ep_p2p_combine(int T, int H, int topk, int E, const void* workspace, const nvfp4b_ep_peers* peers,
                          float* out, int flags, void* stream);

/* nvfp4b_ep_p2p_combine plus the chained outputs of nvfp4b_moe_forward_chain (bf16 copy of the finished rows into
 * x_next, their max |.| into *d_amax_next, zeroed by this call). */
int nvfp4b_ep_p2p_combine_chain(int T, int H, int topk, int E, const void* workspace, const nvfp4b_ep_peers* peers,
                                float* out, int flags, void* x_next, float* d_amax_next, void* stream);

/* Router + one expert-parallel layer on this rank in one call: nvfp4b_moe_route over all E experts (proj [E, H]),
 * nvfp4b_ep_p2p_dispatch, nvfp4b_ep_p2p_expert_forward (local_experts: this rank's E / G) and
 * nvfp4b_ep_p2p_combine (x_next / d_amax_next NULL) or _combine_chain (both given), with the same results, and with
 * the router top-k sharing its kernel with the dispatch ranking and the chained amax reset inside the down GEMM (no
 * memset).  ids / weights [T, topk] receive the routing; src_workspace / exp_workspace as for the dispatch and the
 * expert side.  flags: NVFP4B_MOE_ACCUMULATE or 0. */
int nvfp4b_ep_p2p_layer(const void* x, int T, const void* proj, int topk, const float* per_expert_scale, int norm,
                        int E, const nvfp4b_moe_experts* local_experts, float in_gscale, const float* d_in_amax,
                        float* out, int flags, int* ids, float* weights, void* src_workspace, void* exp_workspace,
                        const nvfp4b_ep_peers* peers, int* overflow, void* x_next, float* d_amax_next, void* stream);

/* Bound of every wait on another rank's flag (records landed, rows landed) in kernels launched after this call:
 * ns nanoseconds per flag, 1 us ... 600 s; 0 restores the default of 10 s.  A wait that runs out records
 * NVFP4B_ERR_TIMEOUT's device code (nvfp4b_read_device_error() == 4) and its kernel goes on; the exchange's layer
 * epochs are then out of step between the ranks, so the exchange buffers must be created anew before the next
 * layer.  A CUDA graph keeps the bound its kernels were captured with.  Host-side setting, no CUDA call. */
int nvfp4b_ep_set_peer_wait_ns(unsigned long long ns);

/* Debug reads (synchronous, not for capture): a rank's private words (layer epoch, completion counters, spare) and
 * its receive counts [G] (records from each source in the last layer). */
int nvfp4b_ep_p2p_state(const nvfp4b_ep_peers* peers, unsigned* host_words4);
int nvfp4b_ep_p2p_recv_counts(const nvfp4b_ep_peers* peers, int* host_counts);

/* Set-up helpers (not capture-safe, they allocate or map): a zeroed device allocation whose CUDA IPC handle
 * (64 bytes) another process on the node maps with nvfp4b_ipc_open (peer access enabled lazily). */
int nvfp4b_ipc_alloc(size_t bytes, void** ptr);
int nvfp4b_ipc_free(void* ptr);
int nvfp4b_ipc_handle(void* ptr, void* handle64);
int nvfp4b_ipc_open(const void* handle64, void** ptr);
int nvfp4b_ipc_close(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_B200_H */
