// moe.cu -- MoE top-k grouped expert FFN on sm_100a (router, dispatch, grouped NVFP4 GEMMs, combine).
//
// Replaces the reference's device MoE (src/forward.cu:193-321: k_router_hn/scores/top8, k_moe_invert,
// k_moe_gateup(_grouped), k_moe_down) and its orchestration moe() (src/forward.cu:516-553).  Those kernels are
// W4A16 CUDA-core kernels that re-read every expert weight row per (token, slot); here the work is regrouped by
// expert so each weight tile is read once per 128 routed rows and multiplied on the FP4 tensor cores:
//
//   1. router     logits = x @ proj^T: bf16 tcgen05 GEMM (kind::f16) split 4 ways along K into fp32 partials;
//                 one warp per token sums the partials in a fixed order, softmax, top-k (ties -> lower id),
//                 renormalise, x per_expert_scale (src/forward.cu:202-231 semantics).
//   2. dispatch   a deterministic counting sort of the T*k assignments by expert: per-chunk histograms, a plan
//                 kernel (segment starts padded to 128 rows, row-block -> expert map), and a stable rank kernel
//                 (warp match + per-warp counts, so rows keep token order).  Replaces k_moe_invert's atomics and
//                 its 16-row cap.
//   3. quantise   each token row is NVFP4-quantised ONCE and its codes/scales are stored to its k destination
//                 rows (the quantiser fused into the dispatch permutation).
//   4. gate/up    grouped NVFP4 GEMM (gemm_core.cuh, grouped scheduler) over the expert-sorted rows; w13 rows
//                 interleave gate and up in groups of 16 so each 32-column accumulator chunk holds 16 gate and the
//                 matching 16 up columns; the epilogue forms gelu_tanh(gate) * up and requantises it to NVFP4 in
//                 the layout the down GEMM reads (codes + tile-layout scales), with the expert's static scale.
//   5. down       grouped NVFP4 GEMM; the epilogue multiplies each row by its router weight and stores it (fp32)
//                 in an assignment-major buffer; a combine kernel sums each token's k rows in slot order, so the
//                 output is bit-reproducible (an atomic-add variant exists, but the L2's fp32 atomic rate makes
//                 it slower at these sizes).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "gemm_core.cuh"
#include "sm100.cuh"

namespace nvfp4b {
namespace {

constexpr int kRouterMaxSplits = 16;

// Most split-K slices the router GEMM may use for T tokens x E experts: 16, or fewer so the fp32 partials stay
// within 4 MiB (at least 4).  The workspace holds this many [T, E] partial slices.
inline int router_max_splits(int T, int E) {
    const long long te = (long long)T * E;
    const long long fit = te > 0 ? (1ll << 20) / te : kRouterMaxSplits;
    return (int)(fit < 4 ? 4 : fit > kRouterMaxSplits ? kRouterMaxSplits : fit);
}
constexpr int kChunk = 256;           // assignments per histogram / rank chunk (one rank round per CTA)

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

int max_rows_for(int T, int E, int topk) {
    const long long r = (long long)T * topk + (long long)E * 127;
    return (int)((r + 127) / 128 * 128);
}

struct Workspace {
    float* partial;
    int* hist;
    int* chunk_base;
    int* seg_start;
    int* seg_count;
    int* m_tiles;
    int* tile_expert;
    int* dest;
    int* lrank;           // [T*topk] stable rank of each assignment among its chunk's assignments to the same expert
    int* row_token;
    float* row_weight;
    int* row_assign;
    uint16_t* y;          // [T*topk, H] fp16 weighted expert outputs, assignment-major (deterministic combine)
    float* row_gscale;    // [max_rows] per-row activation global scale (expert-parallel rows come from many ranks)
    int* ep_ids;          // [T*topk] expert-parallel: local expert of each received record (expert side),
                          //   record slot of each assignment (source side)
    float* ep_w;          // [T*topk] expert-parallel: router weight of each received record
    int* ep_send;         // [256] expert-parallel over peer memory: records per destination rank (source side)
    uint8_t* a_codes;
    uint8_t* a_scales;
    uint8_t* h_codes;
    uint8_t* h_scales;
    size_t bytes;
};

// Chunks of the dispatch ranking: kChunk assignments (ids given), or the tokens of one block of the fused router
// top-k, at least 8 (one per warp; router_topk_tpw).
inline int max_chunks(int T, int topk) {
    const int a = (T * topk + kChunk - 1) / kChunk, b = (T + 7) / 8;
    return a > b ? a : b;
}

// Tokens per warp of the fused router top-k: one (the most parallel) unless that makes more than two blocks of 8
// warps per SM; then 2, 4, ... while a block's chunk of 8 * tpw * topk assignments stays within 256.
inline int router_topk_tpw(int T, int topk, int sms) {
    int tpw = 1;
    while (16 * tpw * topk <= 256 && (T + 8 * tpw - 1) / (8 * tpw) > 2 * sms) tpw *= 2;
    return tpw;
}

Workspace carve(void* base, int T, int H, int I, int E, int topk) {
    Workspace w{};
    const int n_assign = T * topk;
    const int n_chunks = max_chunks(T, topk);
    const int rows = max_rows_for(T, E, topk);
    char* p = static_cast<char*>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) { char* q = p ? p + off : nullptr; off += align256(bytes); return q; };
    w.partial = (float*)take((size_t)router_max_splits(T, E) * T * E * 4);
    w.hist = (int*)take((size_t)n_chunks * E * 4);
    w.chunk_base = (int*)take((size_t)n_chunks * E * 4);
    w.seg_start = (int*)take((size_t)E * 4);
    w.seg_count = (int*)take((size_t)E * 4);
    w.m_tiles = (int*)take(4);
    w.tile_expert = (int*)take((size_t)(rows / 128) * 4);
    w.dest = (int*)take((size_t)n_assign * 4);
    w.lrank = (int*)take((size_t)n_assign * 4);
    w.row_token = (int*)take((size_t)rows * 4);
    w.row_weight = (float*)take((size_t)rows * 4);
    w.row_assign = (int*)take((size_t)rows * 4);
    w.y = (uint16_t*)take((size_t)n_assign * H * 2);
    w.row_gscale = (float*)take((size_t)rows * 4);
    w.ep_ids = (int*)take((size_t)n_assign * 4);
    w.ep_w = (float*)take((size_t)n_assign * 4);
    w.ep_send = (int*)take(256 * 4);
    w.a_codes = (uint8_t*)take((size_t)rows * (H / 2));
    w.a_scales = (uint8_t*)take(scale_bytes(rows, H));
    w.h_codes = (uint8_t*)take((size_t)rows * (I / 2));
    w.h_scales = (uint8_t*)take(scale_bytes(rows, I));
    w.bytes = off;
    return w;
}

// ---------------------------------------------------------------------------------------------------------------
// 1. router
// ---------------------------------------------------------------------------------------------------------------

struct RouterEpi {
    float* partial;          // [splits][T][E]
    long long split_stride;  // T * E
    int T, E;
    __device__ __forceinline__ void finish() const {}
    __device__ __forceinline__ bool row_live(const TileInfo&, int) const { return true; }
    template <int CH>
    __device__ __forceinline__ void process(const TileInfo& ti, int row, int col_base, const uint32_t (&r)[CH][32],
                                            uint8_t*) const {
        const int m = ti.a_row + row;
        if (m >= T) return;
        float* dst = partial + ti.split * split_stride + (long long)m * E;
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int n0 = ti.n0 + col_base + 32 * c;
            if (n0 >= E) continue;
#pragma unroll
            for (int v = 0; v < 8; ++v)
                *reinterpret_cast<float4*>(dst + n0 + 4 * v) =
                    make_float4(__uint_as_float(r[c][4 * v]), __uint_as_float(r[c][4 * v + 1]),
                                __uint_as_float(r[c][4 * v + 2]), __uint_as_float(r[c][4 * v + 3]));
        }
    }
};

using RouterCfg = KCfg<128, 6, 2, 4, Kind::BF16>;

// Top-k of token t, one warp: sum of the split-K partial logits in split order (every split's loads issued before
// the first add), optional per-token norm factor, softmax over E experts, top-k with ties to the lower id,
// renormalised and times per_expert_scale.  Lane j < topk returns the j-th choice in *id / *wt (other lanes: -1).
template <int EPL>
__device__ __forceinline__ void route_token(const float* __restrict__ partial, int splits, long long split_stride,
                                            int t, int E, int topk, const uint16_t* __restrict__ xnorm, int H,
                                            const float* __restrict__ pes, int lane, int* id, float* wt) {
    float l[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) l[i] = 0.f;
    const float* pt = partial + (long long)t * E + lane;
    float v[kRouterMaxSplits][EPL];
#pragma unroll
    for (int u = 0; u < kRouterMaxSplits; ++u)
#pragma unroll
        for (int i = 0; i < EPL; ++i) v[u][i] = u < splits ? __ldg(pt + u * split_stride + 32 * i) : 0.f;
#pragma unroll
    for (int u = 0; u < kRouterMaxSplits; ++u)
#pragma unroll
        for (int i = 0; i < EPL; ++i)
            if (u < splits) l[i] += v[u][i];
    if (xnorm) {   // reference k_router_hn: x * rsqrt(mean(x^2) + 1e-6) * H^-0.5 (scale folded into proj)
        const uint16_t* xr = xnorm + (long long)t * H;
        float ss = 0.f;
        for (int k = lane * 8; k < H; k += 256) {
            const uint4 q = __ldg(reinterpret_cast<const uint4*>(xr + k));
            const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float a = bf16lo(w4[i]), b = bf16hi(w4[i]);
                ss = fmaf(a, a, ss);
                ss = fmaf(b, b, ss);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        const float f = rsqrtf(ss / (float)H + 1e-6f) * rsqrtf((float)H);
#pragma unroll
        for (int i = 0; i < EPL; ++i) l[i] *= f;
    }
    float mx = l[0];
#pragma unroll
    for (int i = 1; i < EPL; ++i) mx = fmaxf(mx, l[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    float p[EPL], sum = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) { p[i] = expf(l[i] - mx); sum += p[i]; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
#pragma unroll
    for (int i = 0; i < EPL; ++i) p[i] = p[i] / sum;
    unsigned used = 0u;
    int my_id = -1;
    float my_p = 0.f, wsum = 0.f;
    for (int j = 0; j < topk; ++j) {
        float bv = -1.f;
        int be = 0x7FFFFFFF;
#pragma unroll
        for (int i = 0; i < EPL; ++i)
            if (!((used >> i) & 1u) && p[i] > bv) { bv = p[i]; be = lane + 32 * i; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
            const int oe = __shfl_xor_sync(0xFFFFFFFFu, be, o);
            if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
        }
        if ((be & 31) == lane) used |= 1u << (be >> 5);
        if (lane == j) { my_id = be; my_p = bv; }
        wsum += bv;
    }
    float w = 0.f;
    if (lane < topk) {
        w = my_p / wsum;
        if (pes) w *= __ldg(pes + my_id);
    }
    *id = my_id;
    *wt = w;
}

template <int EPL>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ partial, int splits,
                                                          long long split_stride, int T, int E, int topk,
                                                          const uint16_t* __restrict__ xnorm, int H,
                                                          const float* __restrict__ pes, int* __restrict__ ids,
                                                          float* __restrict__ wout) {
    const int lane = threadIdx.x & 31;
    const int t = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (t >= T) return;
    int id;
    float w;
    route_token<EPL>(partial, splits, split_stride, t, E, topk, xnorm, H, pes, lane, &id, &w);
    if (lane < topk) {
        ids[(long long)t * topk + lane] = id;
        wout[(long long)t * topk + lane] = w;
    }
}

// ---------------------------------------------------------------------------------------------------------------
// 2. dispatch
// ---------------------------------------------------------------------------------------------------------------

// Called by all 256 threads of a block that owns one chunk of at most 256 assignments (thread i: assignment i of the
// chunk, expert e, or -1 for none): writes the chunk's histogram hist[chunk][e] and the stable rank of every
// assignment among the chunk's earlier assignments to the same expert (lrank; warps in order, lanes in order), so
// that the final row of assignment a is chunk_base[chunk][e] + lrank[a] once the plan kernel has laid out the
// segments.  Assignments with an id outside [0, E) get lrank -1 (they are dropped).
__device__ __forceinline__ void chunk_hist_rank(int e, long long a, bool valid, int E, int chunk,
                                                int* __restrict__ hist, int* __restrict__ lrank) {
    __shared__ int wcnt[8][256];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < 8 * 256; i += 256) (&wcnt[0][0])[i] = 0;
    if (!(e >= 0 && e < E)) e = -1;
    __syncthreads();
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(peers);
    __syncthreads();
    if (valid) {
        int r = -1;
        if (e >= 0) {
            r = rank;
            for (int q = 0; q < warp; ++q) r += wcnt[q][e];
        }
        lrank[a] = r;
    }
    for (int i = tid; i < E; i += 256) {
        int c = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) c += wcnt[q][i];
        hist[(long long)chunk * E + i] = c;
    }
}

// ids given: one chunk of kChunk assignments per block.
__global__ void __launch_bounds__(256) moe_hist_rank_kernel(const int* __restrict__ ids, int n_assign, int E,
                                                            int* __restrict__ hist, int* __restrict__ lrank) {
    static_assert(kChunk == 256, "one assignment per thread");
    const long long a = (long long)blockIdx.x * kChunk + threadIdx.x;
    const bool valid = a < n_assign;
    chunk_hist_rank(valid ? __ldg(ids + a) : -1, a, valid, E, blockIdx.x, hist, lrank);
}

// The router's top-k fused with the dispatch ranking: a block routes tpb = 8 * tpw consecutive tokens (warp w takes
// tokens w, w + 8, ...), so its tpb * topk (<= 256) assignments are one chunk, which it then ranks and counts as
// moe_hist_rank_kernel does (chunk size tpb * topk instead of kChunk).
template <int EPL>
__global__ void __launch_bounds__(256) router_topk_rank_kernel(const float* __restrict__ partial, int splits,
                                                               long long split_stride, int T, int E, int topk,
                                                               const uint16_t* __restrict__ xnorm, int H,
                                                               const float* __restrict__ pes, int* __restrict__ ids,
                                                               float* __restrict__ wout, int* __restrict__ hist,
                                                               int* __restrict__ lrank, int tpw) {
    __shared__ int s_ids[256];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tpb = 8 * tpw;
    const int t0 = blockIdx.x * tpb;
    for (int lt = warp; lt < tpb; lt += 8) {
        const int t = t0 + lt;
        int id = -1;
        float w = 0.f;
        if (t < T) route_token<EPL>(partial, splits, split_stride, t, E, topk, xnorm, H, pes, lane, &id, &w);
        if (lane < topk) {
            s_ids[lt * topk + lane] = id;
            if (t < T) {
                ids[(long long)t * topk + lane] = id;
                wout[(long long)t * topk + lane] = w;
            }
        }
    }
    __syncthreads();
    const int n = min(tpb, T - t0) * topk;
    const bool valid = (int)threadIdx.x < n;
    chunk_hist_rank(valid ? s_ids[threadIdx.x] : -1, (long long)t0 * topk + threadIdx.x, valid, E, blockIdx.x,
                    hist, lrank);
}

// Segment layout from the chunk histograms, one block of kPlanThreads: 4 threads per expert (E <= 256), thread q of
// expert e owning the q-th quarter of the chunks, so the histogram column is read with 4-way parallelism and a few
// loads in flight per thread.  seg_count[e] = total rows of e; seg_start[e] = start of its segment (segments padded
// to 128 rows, in expert order); chunk_base[c][e] = seg_start[e] + rows of e in chunks before c; tile_expert[] and
// *m_tiles describe the 128-row blocks for the grouped GEMM scheduler.
constexpr int kPlanThreads = 1024;
__global__ void __launch_bounds__(kPlanThreads) moe_plan_kernel(const int* __restrict__ hist, int n_chunks, int E,
                                                                int* __restrict__ chunk_base,
                                                                int* __restrict__ seg_start,
                                                                int* __restrict__ seg_count, int* __restrict__ m_tiles,
                                                                int* __restrict__ tile_expert) {
    __shared__ int part[4][256];
    __shared__ int padded[257];
    __shared__ int wsum[8];
    const int e = threadIdx.x & 255, q = threadIdx.x >> 8;
    const int per = (n_chunks + 3) / 4;
    const int c0 = q * per, c1 = min(n_chunks, c0 + per);
    int sum = 0;
    if (e < E) {
        int c = c0;
        for (; c + 4 <= c1; c += 4) {
            const int h0 = __ldg(hist + (long long)c * E + e), h1 = __ldg(hist + (long long)(c + 1) * E + e);
            const int h2 = __ldg(hist + (long long)(c + 2) * E + e), h3 = __ldg(hist + (long long)(c + 3) * E + e);
            sum += (h0 + h1) + (h2 + h3);
        }
        for (; c < c1; ++c) sum += __ldg(hist + (long long)c * E + e);
    }
    part[q][e] = sum;
    __syncthreads();
    const int total = part[0][e] + part[1][e] + part[2][e] + part[3][e];
    if (q == 0) {   // inclusive scan of the padded segment sizes -> padded[e + 1] = end of segment e
        const int lane = e & 31, wid = e >> 5;
        int v = (e < E) ? (total + 127) / 128 * 128 : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xFFFFFFFFu, v, o);
            if (lane >= o) v += u;
        }
        if (lane == 31) wsum[wid] = v;
        padded[e + 1] = v;      // within the warp; the earlier warps' totals are added below
        if (e == 0) padded[0] = 0;
    }
    __syncthreads();
    if (q == 0) {
        int off = 0;
        for (int w = 0; w < (e >> 5); ++w) off += wsum[w];
        padded[e + 1] += off;
    }
    __syncthreads();
    if (e < E) {
        const int start = padded[e];
        if (q == 0) {
            seg_start[e] = start;
            seg_count[e] = total;
        }
        int run = start;
        for (int qq = 0; qq < q; ++qq) run += part[qq][e];
        for (int c = c0; c < c1; ++c) {
            chunk_base[(long long)c * E + e] = run;
            run += __ldg(hist + (long long)c * E + e);
        }
        for (int r = start + 128 * q; r < padded[e + 1]; r += 512) tile_expert[r / 128] = e;
    }
    if (threadIdx.x == 0) *m_tiles = padded[E] / 128;
}

// ---------------------------------------------------------------------------------------------------------------
// 3. quantise once, scatter to every destination row
// ---------------------------------------------------------------------------------------------------------------

constexpr int kScatterWarps = 6;   // warps per token in the quantise-and-scatter kernel (6 x 32 lanes >= H/16 = 176)

// kScatterWarps warps per token: warp `part` quantises every kScatterWarps-th run of 32 blocks of x[t] once and
// writes each block to all of the token's destination rows.  The destination row of assignment a = t * topk + j is
// chunk_base[a / chunk][e] + lrank[a] (e = ids[a]; the plan kernel laid out the segments, the ranking kernel ranked
// the chunk of `chunk` assignments); warp 0 of the token also records the row's metadata (dest, token, weight,
// assignment).  Rows of segment padding are not written at all: the GEMM epilogues tell them apart by the segment
// bounds, and a padding row's products (whatever its stale codes and scales) land only in that row's outputs, which
// are never stored.  With norm_w (bf16 [H]) the row is RMS-normalised first, x * rsqrt(mean(x^2) + eps) * norm_w in
// fp32 (the reference's rmsnorm, kernels/elementwise.cu:10-22, applied to the MoE input as pre_feedforward_layernorm_2
// in src/forward.cu:535), and the fp32 values are quantised: the normalised activations are never stored.
__global__ void __launch_bounds__(256) moe_quant_scatter_kernel(const uint16_t* __restrict__ x, int T, int H,
                                                                int topk, const int* __restrict__ ids,
                                                                const float* __restrict__ weights, int E,
                                                                const int* __restrict__ chunk_base,
                                                                const int* __restrict__ lrank, int chunk,
                                                                int* __restrict__ dest, int* __restrict__ row_token,
                                                                float* __restrict__ row_weight,
                                                                int* __restrict__ row_assign,
                                                                float gscale, const float* __restrict__ d_amax,
                                                                uint8_t* __restrict__ a_codes,
                                                                uint8_t* __restrict__ a_scales, int tile_cols,
                                                                const uint16_t* __restrict__ norm_w, float eps) {
    const int lane = threadIdx.x & 31;
    const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int t = gw / kScatterWarps, part = gw % kScatterWarps;
    if (t >= T) return;
    const float g = d_amax ? gscale_from_amax(__ldg(d_amax)) : gscale;
    int my_dest = -1;
    if (lane < topk) {
        const int a = t * topk + lane;
        const int e = __ldg(ids + a);
        const int r = __ldg(lrank + a);
        if (e >= 0 && e < E && r >= 0) my_dest = __ldg(chunk_base + (a / chunk) * E + e) + r;
        if (part == 0) {
            dest[a] = my_dest;
            if (my_dest >= 0) {
                row_token[my_dest] = t;
                row_weight[my_dest] = __ldg(weights + a);
                row_assign[my_dest] = a;
            }
        }
    }
    const int kb = H >> 4;
    const uint16_t* xr = x + (long long)t * H;
    float inv = 1.f;
    if (norm_w) {                                    // every warp of the token reduces the whole row (L1-resident)
        float ss = 0.f;
        for (int k = lane * 8; k < H; k += 256) {
            const uint4 q = __ldg(reinterpret_cast<const uint4*>(xr + k));
            const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float a = bf16lo(w4[i]), b = bf16hi(w4[i]);
                ss = fmaf(a, a, ss);
                ss = fmaf(b, b, ss);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        inv = rsqrtf(ss / (float)H + eps);
    }
    for (int b0 = part * 32; b0 < kb; b0 += 32 * kScatterWarps) {
        const int b = b0 + lane;
        uint32_t w0 = 0, w1 = 0, sf = 0;
        if (b < kb) {
            const uint4 q0 = __ldg(reinterpret_cast<const uint4*>(xr + b * 16));
            const uint4 q1 = __ldg(reinterpret_cast<const uint4*>(xr + b * 16) + 1);
            const uint32_t ww[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            if (norm_w) {
                const uint4 n0 = __ldg(reinterpret_cast<const uint4*>(norm_w + b * 16));
                const uint4 n1 = __ldg(reinterpret_cast<const uint4*>(norm_w + b * 16) + 1);
                const uint32_t nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
                float v[16];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    v[2 * i] = __fmul_rn(__fmul_rn(bf16lo(ww[i]), inv), bf16lo(nw[i]));
                    v[2 * i + 1] = __fmul_rn(__fmul_rn(bf16hi(ww[i]), inv), bf16hi(nw[i]));
                }
                sf = quantize16(v, g, w0, w1);
            } else {
                sf = quantize16_bf16(ww, g, w0, w1);
            }
        }
        for (int j = 0; j < topk; ++j) {
            const int r = __shfl_sync(0xFFFFFFFFu, my_dest, j);
            if (r < 0 || b >= kb) continue;
            *reinterpret_cast<uint2*>(a_codes + (long long)r * (H >> 1) + b * 8) = make_uint2(w0, w1);
            a_scales[((long long)(r >> 7) * tile_cols + (b >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 +
                     (b & 3)] = (uint8_t)sf;
        }
    }
}

// ---- peer-memory signalling (expert parallelism without a collective library) ---------------------------------

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bound of every wait on another rank's flag: 10 s by default, settable with nvfp4b_ep_set_peer_wait_ns (read on
// the host when a kernel that waits is launched, and passed to it as an argument).
constexpr unsigned long long kPeerWaitDefaultNs = 10000000000ull;
std::atomic<unsigned long long> g_peer_wait_ns{kPeerWaitDefaultNs};

// Per-rank private words (nvfp4b_ep_peers::state): the epoch of the current layer (advanced by the last block of
// the layer's pack kernel, which publishes the layer's records with it), and the completion counters of the two
// kernels that publish to other ranks.  Every flag of a layer carries its epoch.
enum EpState : int { kEpEpoch = 0, kEpPackDone = 1, kEpDownDone = 2 };

// Source-side publication arguments of ep_pack_kernel (recv == nullptr: local record slots, no publication).
struct EpPackPeers {
    uint8_t* const* recv;
    int* const* counts;
    unsigned* const* flags;
    unsigned* state;
    const int* send_counts;
    int rank, G;
};

// Called by every thread of a block after its last store to peer memory.  The block barrier orders the block's
// stores before thread 0's fence and arrival (GPU scope: the arriving blocks and the last one share the GPU); true
// in every thread of the block that arrives last (the counter is reset for the next launch).  That block's
// system-scope fence then orders every block's stores (cumulatively) before the release stores that follow it.
__device__ __forceinline__ bool last_block_arrived(unsigned* counter) {
    __shared__ unsigned s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned old = atomicAdd(counter, 1u);
        s_last = old == gridDim.x - 1 ? 1u : 0u;
        if (s_last) {
            *counter = 0u;
            __threadfence_system();
        }
    }
    __syncthreads();
    return s_last != 0u;
}

// Thread 0 of a block: waits until flags[g] >= epoch for every g < G (acquire, system scope; bounded by wait_ns
// per flag, after which kErrTimeoutPeer is recorded in *err and the wait ends, and once *err is set no later wait
// spins at all); the block barrier then makes what the flags publish visible to the block.
__device__ __forceinline__ void wait_peer_flags(const unsigned* flags, int G, unsigned epoch, int* err,
                                                unsigned long long wait_ns) {
    if (threadIdx.x == 0) {
        bool ok = true;
        const volatile int* verr = err;
        for (int g = 0; g < G && ok; ++g) {
            if ((int)(ld_acquire_sys(flags + g) - epoch) >= 0) continue;
            const unsigned long long t0 = sm100::globaltimer();
            while ((int)(ld_acquire_sys(flags + g) - epoch) < 0) {
                if (*verr != 0 || sm100::globaltimer() - t0 > wait_ns) { ok = false; break; }
                __nanosleep(64);
            }
        }
        if (!ok) atomicCAS(err, 0, sm100::kErrTimeoutPeer);   // keeps an error recorded earlier
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------------------------------------------
// 4./5. grouped GEMM epilogues
// ---------------------------------------------------------------------------------------------------------------

__device__ __forceinline__ float gelu_tanh(float x) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))   (kernels/elementwise.cu:44-47 of the reference)
    return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

template <bool CALIBRATE>
struct GateUpEpi {
    uint8_t* h_codes;
    uint8_t* h_scales;
    int I, h_tile_cols;
    const float* w1_gscale;
    const float* w3_gscale;
    const float* a2_gscale;
    float in_gscale;
    const float* d_in_amax;
    const float* row_gscale;   // if set: per-row activation global scale (overrides in_gscale / d_in_amax)
    float* h_amax;   // calibration output
    const int* seg_start;      // [E] first row of each expert segment
    const int* seg_count;      // [E] real rows of each expert segment (the rest up to 128 is padding)

    __device__ __forceinline__ void finish() const {}
    // Rows of expert-segment padding hold no token: a warp whose 32 rows are all padding skips its work.
    __device__ __forceinline__ bool row_live(const TileInfo& ti, int row) const {
        return ti.a_row + row - __ldg(seg_start + ti.expert) < __ldg(seg_count + ti.expert);
    }

    template <int CH>
    __device__ __forceinline__ void process(const TileInfo& ti, int row, int col_base, const uint32_t (&r)[CH][32],
                                            uint8_t*) const {
        const int e = ti.expert;
        const long long m = (long long)ti.a_row + row;
        const float gin = row_gscale ? __ldg(row_gscale + m) : d_in_amax ? gscale_from_amax(__ldg(d_in_amax)) : in_gscale;
        const float ag = __frcp_rn(gin * __ldg(w1_gscale + e));
        const float au = __frcp_rn(gin * __ldg(w3_gscale + e));
        const int jb0 = (ti.n0 + col_base) >> 5;          // first 16-wide block of h handled by this thread
        if constexpr (CALIBRATE) {
            float amax = 0.f;
            const bool real = row_live(ti, row);            // padding rows hold no token
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                if ((jb0 + c) * 16 >= I || !real) continue;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float h = gelu_tanh(ag * __uint_as_float(r[c][i])) * (au * __uint_as_float(r[c][16 + i]));
                    amax = fmaxf(amax, fabsf(h));
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
            if ((threadIdx.x & 31) == 0 && amax > 0.f) atomicMax(reinterpret_cast<unsigned*>(h_amax + e), __float_as_uint(amax));
        } else {
            const float g = __ldg(a2_gscale + e);
            uint32_t sfw = 0;
            uint32_t cw[CH][2];
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                float h[16];
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    h[i] = gelu_tanh(ag * __uint_as_float(r[c][i])) * (au * __uint_as_float(r[c][16 + i]));
                const uint32_t sf = quantize16(h, g, cw[c][0], cw[c][1]);
                sfw |= sf << (8 * c);
            }
            uint8_t* dst = h_codes + m * (I >> 1) + jb0 * 8;
            const long long soff = ((m >> 7) * h_tile_cols + (jb0 >> 2)) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4;
            if (CH == 4 && (jb0 + 4) * 16 <= I) {
                *reinterpret_cast<uint4*>(dst) = make_uint4(cw[0][0], cw[0][1], cw[1][0], cw[1][1]);
                *reinterpret_cast<uint4*>(dst + 16) = make_uint4(cw[2][0], cw[2][1], cw[3][0], cw[3][1]);
                *reinterpret_cast<uint32_t*>(h_scales + soff) = sfw;
            } else {
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    const int jb = jb0 + c;
                    if (jb * 16 >= I) continue;
                    *reinterpret_cast<uint2*>(dst + 8 * c) = make_uint2(cw[c][0], cw[c][1]);
                    h_scales[((m >> 7) * h_tile_cols + (jb >> 2)) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 +
                             (jb & 3)] = (uint8_t)(sfw >> (8 * c));
                }
            }
        }
    }
};

// f32 pair -> f16x2 (round to nearest, saturating to +-65504 instead of overflowing), lo in the low half.
__device__ __forceinline__ uint32_t pack_half2_sat(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float2 unpack_half2(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

// Down epilogue.  Row m holds assignment a = token * topk + slot (or -1 for padding); its contribution is
// weight(a) / (g_h * g_w2) * acc.
//   DETERMINISTIC = true (default): stores the row into y[a, :] (assignment-major) as fp16; moe_combine_kernel then
//     sums each token's topk rows in slot order in fp32, giving bit-reproducible output.  fp16 (11-bit significand,
//     relative rounding 2^-11) halves the bytes of the y round trip through HBM, which bounds this stage: y is
//     T * topk * H values (92M for the 4096-token layer), written here and read back once by the combine.
//   DETERMINISTIC = false: adds the fp32 row into out[token, :] with 16-byte vector reductions (order-dependent
//     rounding; bounded by the L2's atomic throughput, so slower at large T*topk).
template <bool DETERMINISTIC>
struct DownEpi {
    uint16_t* y;
    float* out;
    int H, topk;
    const int* row_assign;
    const float* weights;
    const float* w2_gscale;
    const float* a2_gscale;
    const int* seg_start;      // [E] first row of each expert segment
    const int* seg_count;      // [E] real rows of each expert segment (the rest up to 128 is padding)
    // Expert parallelism over peer memory (DETERMINISTIC only): the row of received slot a = s * capacity + j goes
    // to source rank s's return rows, row rank * capacity + j, instead of y[a]; the last epilogue warp of the grid
    // then raises the rows-landed flags (flags[s][G + rank]).
    uint16_t* const* peer_back = nullptr;
    unsigned* const* peer_flags = nullptr;
    unsigned* state = nullptr;
    int rank = 0, G = 0, capacity = 0;
    bool transpose = false;     // rows through the shared-memory transpose (launched with DownTransposeCfg)
    float* zero_word = nullptr; // if set, stored as 0 once by the kernel (the chained amax the combine accumulates)

    // Padding rows of an expert segment produce nothing (their row_assign is never written): a warp whose 32 rows
    // are all padding skips its work.
    __device__ __forceinline__ bool row_live(const TileInfo& ti, int row) const {
        return ti.a_row + row - __ldg(seg_start + ti.expert) < __ldg(seg_count + ti.expert);
    }

    // Every epilogue warp (warps 4.. of every CTA) calls this once after its last tile.
    __device__ __forceinline__ void finish() const {
        if (zero_word && blockIdx.x == 0 && threadIdx.x == 128) *zero_word = 0.0f;
        if constexpr (DETERMINISTIC) {
            if (!peer_back) return;
            __syncwarp();
            if ((threadIdx.x & 31) == 0) {
                __threadfence();                         // arrival at GPU scope; the last warp fences system-wide
                const unsigned total = gridDim.x * ((blockDim.x >> 5) - 4u);
                if (atomicAdd(state + kEpDownDone, 1u) == total - 1u) {
                    state[kEpDownDone] = 0u;
                    __threadfence_system();
                    const unsigned epoch = state[kEpEpoch];
                    for (int g = 0; g < G; ++g) st_release_sys(peer_flags[g] + G + rank, epoch);
                }
            }
        }
    }

    // DETERMINISTIC, rows to local memory: each lane converts its row's 32-column chunk to fp16 and stores it as four
    // 16-byte pieces (64 contiguous bytes of the row); no shared-memory transpose, so the epilogue's per-tile cost --
    // which bounds this short-K GEMM -- is a handful of instructions per chunk.
    // DETERMINISTIC with `transpose`: each warp transposes its 32 x 32 chunk through shared memory as fp16, 16 rows
    // at a time (16 x 17 words per warp, the EPI_SMEM of DownTransposeCfg: small enough to keep 4 pipeline stages;
    // a 32 x 33 fp32 tile left room for 3 only, which cost the kernel 4-10 us), and every store instruction writes
    // eight whole 64-byte row segments.
    // Used for rows to peer memory (16-byte pieces of 32 different rows per instruction cost NVLink packets of half a
    // 32-byte sector each) and for large row counts (the row buffer then streams to DRAM, where scattered 16-byte
    // pieces cost more than the transpose: 125 vs 105 us for 32768 rows of 2816).
    template <int CH>
    __device__ __forceinline__ void process(const TileInfo& ti, int row, int col_base, const uint32_t (&r)[CH][32],
                                            uint8_t* esm) const {
        const long long m = (long long)ti.a_row + row;
        const int a = row_live(ti, row) ? __ldg(row_assign + m) : -1;
        const int e = ti.expert;
        const float s = a >= 0 ? __ldg(weights + a) * __frcp_rn(__ldg(a2_gscale + e) * __ldg(w2_gscale + e)) : 0.f;
        if constexpr (DETERMINISTIC) {
            if (transpose) {
                const int lane = threadIdx.x & 31;
                uint16_t* rowp = a < 0 ? nullptr
                                 : peer_back ? peer_back[a / capacity] + ((long long)rank * capacity + a % capacity) * H
                                             : y + (long long)a * H;
                // per warp a 16-row x 17-word tile of fp16 pairs (the padding word spreads a column over the banks):
                // the warp's 32 rows go through it in two halves of 16; in each of two rounds per half, lane
                // (g, q) = (lane / 4, lane % 4) stores 16 bytes (columns 8q..8q+7) of row 8k + g of the half, so one
                // store instruction writes whole 64-byte segments of 8 rows
                uint32_t* tile = reinterpret_cast<uint32_t*>(esm) + ((threadIdx.x >> 5) - 4) * (16 * 17);   // warps 4..
                const int g = lane >> 2, q = lane & 3;
                uint16_t* prow[2][2];      // the row this lane stores in round k of half h (same for every chunk)
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int k = 0; k < 2; ++k)
                        prow[h][k] = reinterpret_cast<uint16_t*>(__shfl_sync(
                            0xFFFFFFFFu, reinterpret_cast<unsigned long long>(rowp), 16 * h + 8 * k + g));
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    const int n0 = ti.n0 + col_base + 32 * c;   // warp-uniform
                    if (n0 >= H) continue;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        __syncwarp();
                        if ((lane >> 4) == h)
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                tile[(lane & 15) * 17 + i] = pack_half2_sat(s * __uint_as_float(r[c][2 * i]),
                                                                            s * __uint_as_float(r[c][2 * i + 1]));
                        __syncwarp();
#pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            const int lr = 8 * k + g;
                            uint16_t* pi = prow[h][k];
                            const uint32_t* src = tile + lr * 17 + 4 * q;
                            if (pi) *reinterpret_cast<uint4*>(pi + n0 + 8 * q) = make_uint4(src[0], src[1], src[2], src[3]);
                        }
                    }
                }
                return;
            }
            if (a < 0) return;
            uint16_t* rowp = y + (long long)a * H;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int n0 = ti.n0 + col_base + 32 * c;
                if (n0 >= H) continue;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint4 v;
                    v.x = pack_half2_sat(s * __uint_as_float(r[c][8 * q + 0]), s * __uint_as_float(r[c][8 * q + 1]));
                    v.y = pack_half2_sat(s * __uint_as_float(r[c][8 * q + 2]), s * __uint_as_float(r[c][8 * q + 3]));
                    v.z = pack_half2_sat(s * __uint_as_float(r[c][8 * q + 4]), s * __uint_as_float(r[c][8 * q + 5]));
                    v.w = pack_half2_sat(s * __uint_as_float(r[c][8 * q + 6]), s * __uint_as_float(r[c][8 * q + 7]));
                    *reinterpret_cast<uint4*>(rowp + n0 + 8 * q) = v;
                }
            }
        } else {
            if (a < 0) return;
            float* dst = out + (long long)(a / topk) * H;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int n0 = ti.n0 + col_base + 32 * c;
                if (n0 >= H) continue;
#pragma unroll
                for (int v = 0; v < 8; ++v)
                    atomicAdd(reinterpret_cast<float4*>(dst + n0 + 4 * v),
                              make_float4(s * __uint_as_float(r[c][4 * v]), s * __uint_as_float(r[c][4 * v + 1]),
                                          s * __uint_as_float(r[c][4 * v + 2]), s * __uint_as_float(r[c][4 * v + 3])));
            }
        }
    }
};

// Optional second output of the combine kernels, for a stack of layers on a residual stream: the finished row
// rounded to bf16 (RNE) into x (the next layer's input) and max |x| into *amax (its dynamic activation scale, a
// float ordered by its bit pattern; zeroed by the host entry just before the combine).  x == nullptr: off.
struct CombineNext {
    uint16_t* x;
    float* amax;
};

// Every thread of the block calls this (it ends with a block barrier when nx.x is set).
__device__ __forceinline__ void combine_next(const CombineNext& nx, bool valid, long long off, const float (&acc)[8]) {
    if (!nx.x) return;                               // kernel-uniform
    uint32_t m = 0;
    if (valid) {
        uint32_t b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
            b[i] = *reinterpret_cast<const uint32_t*>(&h);
            m = __vmaxu2(m, b[i] & 0x7FFF7FFFu);
        }
        *reinterpret_cast<uint4*>(nx.x + off) = make_uint4(b[0], b[1], b[2], b[3]);
    }
    __shared__ uint32_t red[32];
    uint32_t m16 = max(m & 0xFFFFu, m >> 16);
    m16 = __reduce_max_sync(0xFFFFFFFFu, m16);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m16;
    __syncthreads();
    if (threadIdx.x < 32) {                          // one atomic per block (same-address atomics serialise)
        uint32_t v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0u;
        v = __reduce_max_sync(0xFFFFFFFFu, v);
        if (threadIdx.x == 0 && v != 0) atomicMax(reinterpret_cast<unsigned*>(nx.amax), v << 16);
    }
}

// out[t] (+)= sum_j y[t*k + j] over the k slots in order, fp32 accumulation of the fp16 rows.  One thread per
// (token, 8 columns): T * H / 8 independent 16-byte gathers; H % 8 == 0.
__global__ void __launch_bounds__(256) moe_combine_kernel(const uint16_t* __restrict__ y, int T, int H, int topk,
                                                          float* __restrict__ out, int accumulate,
                                                          const CombineNext next) {
    const int chunks = H >> 3;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool valid = idx < (long long)T * chunks;
    const int t = valid ? (int)(idx / chunks) : 0, c = valid ? (int)(idx - (long long)t * chunks) * 8 : 0;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    if (valid) {
        const uint16_t* src = y + (long long)t * topk * H + c;
        float* dst = out + (long long)t * H + c;
        if (accumulate) {
            const float4 u = *reinterpret_cast<const float4*>(dst), v = *reinterpret_cast<const float4*>(dst + 4);
            acc[0] = u.x; acc[1] = u.y; acc[2] = u.z; acc[3] = u.w; acc[4] = v.x; acc[5] = v.y; acc[6] = v.z; acc[7] = v.w;
        }
        for (int j = 0; j < topk; ++j) {
            const uint4 q = __ldg(reinterpret_cast<const uint4*>(src + (long long)j * H));
            const float2 f0 = unpack_half2(q.x), f1 = unpack_half2(q.y), f2 = unpack_half2(q.z), f3 = unpack_half2(q.w);
            acc[0] += f0.x; acc[1] += f0.y; acc[2] += f1.x; acc[3] += f1.y;
            acc[4] += f2.x; acc[5] += f2.y; acc[6] += f3.x; acc[7] += f3.y;
        }
        *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    combine_next(next, valid, (long long)t * H + c, acc);
}

// ---------------------------------------------------------------------------------------------------------------
// 6. expert parallelism: records exchanged between ranks (source: route + pack; expert: unpack + GEMMs; source:
//    combine).  Record = [e2m1 codes H/2][logical e4m3 scales H/16][meta: local expert, router weight, activation
//    global scale, 0], 16-byte aligned; a source packs its assignments sorted by expert, i.e. by destination rank
//    (rank = expert / experts_per_rank), so each destination's records are one contiguous run.
// ---------------------------------------------------------------------------------------------------------------

struct EpMeta {
    int expert;      // local expert on the destination rank
    float weight;    // router weight of the assignment
    float gscale;    // activation global scale the codes were made with
    int pad;
};

__host__ __device__ inline size_t ep_record_bytes(int H) { return (size_t)(H / 2) + (size_t)(H / 16) + sizeof(EpMeta); }

// Compact (unpadded) expert-sorted positions: chunk_base[c][e] = first row of expert e's assignments from chunk c;
// dst_start[d] = first position of destination rank d's run; send_counts[d] = records for rank d, at most
// `capacity` (the fixed slot count per destination); more sets *overflow (the excess is not sent).
__global__ void __launch_bounds__(256) ep_plan_kernel(const int* __restrict__ hist, int n_chunks, int E,
                                                      int experts_per_rank, int G, int capacity,
                                                      int* __restrict__ chunk_base, int* __restrict__ seg_count,
                                                      int* __restrict__ dst_start, int* __restrict__ send_counts,
                                                      int* __restrict__ overflow) {
    __shared__ int start[257];
    const int e = threadIdx.x;
    int total = 0;
    if (e < E)
        for (int c = 0; c < n_chunks; ++c) total += hist[c * E + e];
    start[e + 1] = e < E ? total : 0;
    if (e == 0) start[0] = 0;
    __syncthreads();
    if (e == 0)
        for (int i = 1; i <= E; ++i) start[i] += start[i - 1];
    __syncthreads();
    if (e < E) {
        seg_count[e] = total;
        int run = start[e];
        for (int c = 0; c < n_chunks; ++c) {
            chunk_base[c * E + e] = run;
            run += hist[c * E + e];
        }
    }
    if (e < G) {
        const int n = start[min(E, (e + 1) * experts_per_rank)] - start[min(E, e * experts_per_rank)];
        dst_start[e] = start[min(E, e * experts_per_rank)];
        send_counts[e] = min(n, capacity);
        if (n > capacity) atomicOr(overflow, 1);
    }
}

// Warp per token: quantise x[t] once (dynamic or static global scale), write one record per routed slot.
// kPackWarps warps per token, each quantising every kPackWarps-th run of 32 blocks of x[t] and writing them to all
// of the token's records.  slot[a] = d * capacity + (pos - dst_start[d]) for the assignment's destination d, where
// pos = chunk_base[a / chunk][e] + lrank[a] is its compact expert-sorted position, or -1 past the capacity
// (overflowed, not sent).  The record goes to
// records[slot], or with peers.recv to peer d's receive slot rank * capacity + (slot - d * capacity); the last
// block then stores the per-destination counts, raises the records-landed flags and advances the layer epoch.
constexpr int kPackWarps = 6;

__global__ void __launch_bounds__(256) ep_pack_kernel(const uint16_t* __restrict__ x, int T, int H, int topk,
                                                      const int* __restrict__ chunk_base,
                                                      const int* __restrict__ lrank, int chunk, int E,
                                                      const int* __restrict__ ids,
                                                      const float* __restrict__ weights, int experts_per_rank,
                                                      int capacity, const int* __restrict__ dst_start,
                                                      float gscale, const float* __restrict__ d_amax,
                                                      uint8_t* __restrict__ records, int* __restrict__ slot,
                                                      const EpPackPeers peers) {
    const int lane = threadIdx.x & 31;
    const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int t = gw / kPackWarps, part = gw % kPackWarps;
    if (t < T) {
        const float g = d_amax ? gscale_from_amax(__ldg(d_amax)) : gscale;
        const size_t rb = ep_record_bytes(H);
        uint8_t* my_rec = nullptr;
        if (lane < topk) {
            const long long a = (long long)t * topk + lane;
            const int e = __ldg(ids + a), r = __ldg(lrank + a);
            const int pos = (e >= 0 && e < E && r >= 0) ? __ldg(chunk_base + (a / chunk) * E + e) + r : -1;
            int my_slot = -1;
            if (pos >= 0) {
                const int d = __ldg(ids + a) / experts_per_rank;
                const int i = pos - __ldg(dst_start + d);
                if (i < capacity) {
                    my_slot = d * capacity + i;
                    my_rec = peers.recv ? peers.recv[d] + ((size_t)peers.rank * capacity + i) * rb
                                        : records + (size_t)my_slot * rb;
                }
            }
            if (part == 0) {
                slot[a] = my_slot;
                if (my_rec) {
                    EpMeta meta;
                    meta.expert = __ldg(ids + a) % experts_per_rank;
                    meta.weight = __ldg(weights + a);
                    meta.gscale = g;
                    meta.pad = 0;
                    *reinterpret_cast<EpMeta*>(my_rec + (H / 2) + (H / 16)) = meta;
                }
            }
        }
        const int kb = H >> 4;
        const uint16_t* xr = x + (long long)t * H;
        for (int b0 = part * 32; b0 < kb; b0 += 32 * kPackWarps) {
            const int b = b0 + lane;
            uint32_t w0 = 0, w1 = 0, sf = 0;
            if (b < kb) {
                const uint4 q0 = __ldg(reinterpret_cast<const uint4*>(xr + b * 16));
                const uint4 q1 = __ldg(reinterpret_cast<const uint4*>(xr + b * 16) + 1);
                const uint32_t ww[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                sf = quantize16_bf16(ww, g, w0, w1);
            }
            for (int j = 0; j < topk; ++j) {
                uint8_t* rec = reinterpret_cast<uint8_t*>(
                    __shfl_sync(0xFFFFFFFFu, reinterpret_cast<unsigned long long>(my_rec), j));
                if (!rec || b >= kb) continue;
                *reinterpret_cast<uint2*>(rec + b * 8) = make_uint2(w0, w1);
                rec[(H / 2) + b] = (uint8_t)sf;
            }
        }
    }
    if (peers.recv && last_block_arrived(peers.state + kEpPackDone)) {
        const unsigned epoch = peers.state[kEpEpoch] + 1u;     // no other block reads it: all have arrived
        for (int d = threadIdx.x; d < peers.G; d += blockDim.x) {
            peers.counts[d][peers.rank] = peers.send_counts[d];
            st_release_sys(peers.flags[d] + peers.rank, epoch);
        }
        __syncthreads();
        if (threadIdx.x == 0) peers.state[kEpEpoch] = epoch;
    }
}

// Slot i = s * capacity + j holds a record iff j < recv_counts[s]; empty slots get expert -1 (skipped by the plan).
// With wait_flags (exchange over peer memory) every block first waits for the records-landed flags of this layer.
// One block per chunk of kChunk slots: each thread reads its slot's meta, then the block ranks its chunk for the
// dispatch plan (chunk_hist_rank) -- the meta read and the ranking in one launch.
__global__ void __launch_bounds__(256) ep_meta_rank_kernel(const uint8_t* records, int n, int H, int capacity,
                                                           const int* recv_counts, int* __restrict__ ids,
                                                           float* __restrict__ w, int E, int* __restrict__ hist,
                                                           int* __restrict__ lrank, const unsigned* wait_flags, int G,
                                                           const unsigned* state, int* err,
                                                           unsigned long long wait_ns) {
    static_assert(kChunk == 256, "one slot per thread");
    if (wait_flags) wait_peer_flags(wait_flags, G, state[kEpEpoch], err, wait_ns);
    const int i = blockIdx.x * kChunk + threadIdx.x;
    const bool valid = i < n;
    int e = -1;
    if (valid) {
        float wt = 0.f;
        if (i % capacity < recv_counts[i / capacity]) {
            const EpMeta meta =
                *reinterpret_cast<const EpMeta*>(records + (size_t)i * ep_record_bytes(H) + (H / 2) + (H / 16));
            e = meta.expert;
            wt = meta.weight;
        }
        ids[i] = e;
        w[i] = wt;
    }
    chunk_hist_rank(e, i, valid, E, blockIdx.x, hist, lrank);
}

// Warp per received record slot i: its row r = chunk_base[i / kChunk][e] + lrank[i] of the padded expert-sorted
// operand (e = its local expert, -1 for an empty slot), codes to that row, scales to the tile layout, and the row's
// metadata (slot, weight, the activation global scale the codes were made with).
__global__ void __launch_bounds__(256) ep_scatter_kernel(const uint8_t* __restrict__ records, int n, int H,
                                                         const int* __restrict__ ep_ids, const float* __restrict__ ep_w,
                                                         int E, const int* __restrict__ chunk_base,
                                                         const int* __restrict__ lrank, int* __restrict__ dest,
                                                         int* __restrict__ row_assign, float* __restrict__ row_weight,
                                                         uint8_t* __restrict__ a_codes, uint8_t* __restrict__ a_scales,
                                                         float* __restrict__ row_gscale, int tile_cols) {
    const int lane = threadIdx.x & 31;
    const int i = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (i >= n) return;
    const int e = __ldg(ep_ids + i), rk = __ldg(lrank + i);
    const int r = (e >= 0 && e < E && rk >= 0) ? __ldg(chunk_base + (i / kChunk) * E + e) + rk : -1;
    if (lane == 0) dest[i] = r;
    if (r < 0) return;
    const uint8_t* rec = records + (size_t)i * ep_record_bytes(H);
    const int kb = H >> 4;
    for (int b = lane; b < kb; b += 32) {
        *reinterpret_cast<uint2*>(a_codes + (long long)r * (H >> 1) + b * 8) =
            *reinterpret_cast<const uint2*>(rec + b * 8);
        a_scales[((long long)(r >> 7) * tile_cols + (b >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (b & 3)] =
            rec[(H / 2) + b];
    }
    if (lane == 0) {
        row_gscale[r] = reinterpret_cast<const EpMeta*>(rec + (H / 2) + (H / 16))->gscale;
        row_assign[r] = i;
        row_weight[r] = __ldg(ep_w + i);
    }
}

// out[t] (+)= sum_j y_back[slot[t*k + j]] in slot order (fp32 accumulation of the fp16 rows sent back).  One
// thread per (token, 8 columns): T * H / 8 independent gathers.  With wait_flags (exchange over peer memory) every
// block first waits for the rows-landed flags of this layer.
__global__ void __launch_bounds__(256) ep_combine_kernel(const uint16_t* y_back, int T, int H, int topk,
                                                         const int* __restrict__ slot, float* __restrict__ out,
                                                         int accumulate, const unsigned* wait_flags, int G,
                                                         const unsigned* state, int* err,
                                                         unsigned long long wait_ns, const CombineNext next) {
    if (wait_flags) wait_peer_flags(wait_flags, G, state[kEpEpoch], err, wait_ns);
    const int chunks = H >> 3;
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool valid = idx < (long long)T * chunks;
    const int t = valid ? (int)(idx / chunks) : 0, c = valid ? (int)(idx - (long long)t * chunks) * 8 : 0;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    if (valid) {
        float* dst = out + (long long)t * H + c;
        if (accumulate) {
            const float4 u = *reinterpret_cast<const float4*>(dst), v = *reinterpret_cast<const float4*>(dst + 4);
            acc[0] = u.x; acc[1] = u.y; acc[2] = u.z; acc[3] = u.w; acc[4] = v.x; acc[5] = v.y; acc[6] = v.z; acc[7] = v.w;
        }
        for (int j = 0; j < topk; ++j) {
            const int r = __ldg(slot + (long long)t * topk + j);
            if (r < 0) continue;
            const uint4 q = *reinterpret_cast<const uint4*>(y_back + (long long)r * H + c);
            const float2 f0 = unpack_half2(q.x), f1 = unpack_half2(q.y), f2 = unpack_half2(q.z), f3 = unpack_half2(q.w);
            acc[0] += f0.x; acc[1] += f0.y; acc[2] += f1.x; acc[3] += f1.y;
            acc[4] += f2.x; acc[5] += f2.y; acc[6] += f3.x; acc[7] += f3.y;
        }
        *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    combine_next(next, valid, (long long)t * H + c, acc);
}

using GroupCfg = KCfg<256, 4, 1, 8>;
using DownCfg = KCfg<256, 4, 1, 8>;   // K = I is short: the epilogue bounds it (direct fp16 row stores)
using DownTransposeCfg = KCfg<256, 4, 1, 8, Kind::NVF4, 8 * 16 * 17 * 4>;   // + the epilogue's transpose tiles
constexpr int kDownTransposeRows = 16384;   // local row buffers at least this large take the transposed stores

// ---------------------------------------------------------------------------------------------------------------
// host orchestration
// ---------------------------------------------------------------------------------------------------------------

int check_experts(const nvfp4b_moe_experts* ex) {
    if (!ex || !ex->w13 || !ex->w13_scales || !ex->w2 || !ex->w2_scales || !ex->w1_gscale || !ex->w3_gscale ||
        !ex->w2_gscale || !ex->a2_gscale)
        return NVFP4B_ERR_NULL;
    if (ex->num_experts <= 0 || ex->num_experts > 256 || ex->hidden <= 0 || (ex->hidden % 256) ||
        ex->inter <= 0 || (ex->inter % 32))
        return NVFP4B_ERR_SHAPE;
    if (!aligned16(ex->w13) || !aligned16(ex->w13_scales) || !aligned16(ex->w2) || !aligned16(ex->w2_scales))
        return NVFP4B_ERR_ALIGN;
    return NVFP4B_OK;
}

// Dispatch: hist-rank (per chunk of kChunk assignments) -> plan (segment layout, one block) -> quantise-scatter
// (rows from the plan and the chunk ranks, codes and scales of every real row, row metadata).  With ranked = true
// the chunk histograms and ranks are already in the workspace (the fused router top-k wrote them for chunks of
// `chunk` assignments) and the hist-rank launch is skipped.
int dispatch(const void* x, int T, const int* ids, const float* weights, int topk, int H, int E, float in_gscale,
             const float* d_in_amax, const Workspace& w, cudaStream_t s, const uint16_t* norm_w = nullptr,
             float eps = 0.f, bool ranked = false, int chunk = kChunk) {
    const int n_assign = T * topk;
    const int n_chunks = (n_assign + chunk - 1) / chunk;
    int st;
    if (!ranked) {
        st = launch_k(moe_hist_rank_kernel, dim3(n_chunks), dim3(256), 0, s, ids, n_assign, E, w.hist, w.lrank);
        if (st) return st;
    }
    st = launch_k(moe_plan_kernel, dim3(1), dim3(kPlanThreads), 0, s, w.hist, n_chunks, E, w.chunk_base,
                  w.seg_start, w.seg_count, w.m_tiles, w.tile_expert);
    if (st) return st;
    const int tile_cols = (H / 16 + 3) / 4;
    return launch_k(moe_quant_scatter_kernel, dim3((T * kScatterWarps + 7) / 8), dim3(256), 0, s,
                    static_cast<const uint16_t*>(x), T, H, topk, ids, weights, E, w.chunk_base, w.lrank, chunk,
                    w.dest, w.row_token, w.row_weight, w.row_assign, in_gscale, d_in_amax, w.a_codes, w.a_scales,
                    tile_cols, norm_w, eps);
}

template <bool CALIBRATE>
int gate_up(const nvfp4b_moe_experts* ex, int T, int topk, float in_gscale, const float* d_in_amax, float* h_amax,
            const Workspace& w, cudaStream_t s, bool per_row_gscale = false) {
    const int H = ex->hidden, I = ex->inter, E = ex->num_experts;
    const int rows = max_rows_for(T, E, topk);
    CUtensorMap ma, mb;
    int st = make_kmajor_map(&ma, w.a_codes, rows, H / 2, GroupCfg::BM);
    if (st) return st;
    st = make_kmajor_map(&mb, ex->w13, (long long)E * 2 * I, H / 2, GroupCfg::BN);
    if (st) return st;
    CoreParams cp;
    cp.err = device_error_ptr();
    if (!cp.err) return NVFP4B_ERR_CUDA;
    cp.sfa = w.a_scales;
    cp.sfb = ex->w13_scales;
    cp.tile_cols = (H / 16 + 3) / 4;
    cp.k_tiles = (cp.tile_cols + 3) / 4;
    GroupedSched<GroupCfg::BN> sc{};
    sc.d_m_tiles = w.m_tiles;
    sc.tile_expert = w.tile_expert;
    sc.n_tiles = (2 * I + GroupCfg::BN - 1) / GroupCfg::BN;
    sc.group_m = 8;
    sc.n_per_expert = 2 * I;
    sc.b_row_tiles_per_expert = (2 * I + 127) / 128;
    sc.k_tiles = cp.k_tiles;
    GateUpEpi<CALIBRATE> e;
    e.h_codes = w.h_codes;
    e.h_scales = w.h_scales;
    e.I = I;
    e.h_tile_cols = (I / 16 + 3) / 4;
    e.w1_gscale = ex->w1_gscale;
    e.w3_gscale = ex->w3_gscale;
    e.a2_gscale = ex->a2_gscale;
    e.in_gscale = in_gscale;
    e.d_in_amax = d_in_amax;
    e.row_gscale = per_row_gscale ? w.row_gscale : nullptr;
    e.h_amax = h_amax;
    e.seg_start = w.seg_start;
    e.seg_count = w.seg_count;
    return launch_core<GroupCfg>(ma, mb, cp, sc, e, sm_count(), s);
}

int down(const nvfp4b_moe_experts* ex, int T, int topk, const float* weights, float* out, int flags,
         const Workspace& w, cudaStream_t s, const nvfp4b_ep_peers* peers = nullptr,
         const CombineNext next = CombineNext{nullptr, nullptr}, float* zero_word = nullptr) {
    const bool accumulate = (flags & NVFP4B_MOE_ACCUMULATE) != 0;
    const bool deterministic = (flags & NVFP4B_MOE_ATOMIC) == 0;
    const int H = ex->hidden, I = ex->inter, E = ex->num_experts;
    const int rows = max_rows_for(T, E, topk);
    CUtensorMap ma, mb;
    int st = make_kmajor_map(&ma, w.h_codes, rows, I / 2, DownCfg::BM);
    if (st) return st;
    st = make_kmajor_map(&mb, ex->w2, (long long)E * H, I / 2, DownCfg::BN);
    if (st) return st;
    CoreParams cp;
    cp.err = device_error_ptr();
    if (!cp.err) return NVFP4B_ERR_CUDA;
    cp.sfa = w.h_scales;
    cp.sfb = ex->w2_scales;
    cp.tile_cols = (I / 16 + 3) / 4;
    cp.k_tiles = (cp.tile_cols + 3) / 4;
    GroupedSched<DownCfg::BN> sc{};
    sc.d_m_tiles = w.m_tiles;
    sc.tile_expert = w.tile_expert;
    sc.n_tiles = (H + DownCfg::BN - 1) / DownCfg::BN;
    sc.group_m = 8;
    sc.n_per_expert = H;
    sc.b_row_tiles_per_expert = (H + 127) / 128;
    sc.k_tiles = cp.k_tiles;
    if (deterministic) {
        DownEpi<true> e{w.y, out, H, topk, w.row_assign, weights, ex->w2_gscale, ex->a2_gscale, w.seg_start,
                        w.seg_count};
        if (peers) {
            e.peer_back = peers->back;
            e.peer_flags = peers->flags;
            e.state = peers->state;
            e.rank = peers->rank;
            e.G = peers->G;
            e.capacity = peers->capacity;
        }
        e.transpose = peers != nullptr || (long long)T * topk >= kDownTransposeRows;
        // the chained amax is zeroed by the down kernel: every reader of the layer's input scale (the dispatch and
        // the gate/up epilogue) has finished by then, and the combine that accumulates it runs after
        e.zero_word = (out && next.x) ? next.amax : zero_word;
        static_assert(DownTransposeCfg::BM == DownCfg::BM && DownTransposeCfg::BN == DownCfg::BN, "same tiles, maps");
        st = e.transpose ? launch_core<DownTransposeCfg>(ma, mb, cp, sc, e, sm_count(), s)
                         : launch_core<DownCfg>(ma, mb, cp, sc, e, sm_count(), s);
        if (st || !out) return st;                  // out == nullptr: leave the weighted rows in w.y
        moe_combine_kernel<<<(unsigned)(((long long)T * (H / 8) + 255) / 256), 256, 0, s>>>(w.y, T, H, topk, out,
                                                                                      accumulate ? 1 : 0, next);
        return launch_status();
    }
    if (!accumulate) {
        cudaError_t err = cudaMemsetAsync(out, 0, (size_t)T * H * sizeof(float), s);
        if (err != cudaSuccess) return record_cuda_error(err);
    }
    DownEpi<false> e{w.y, out, H, topk, w.row_assign, weights, ex->w2_gscale, ex->a2_gscale, w.seg_start,
                     w.seg_count};
    return launch_core<DownCfg>(ma, mb, cp, sc, e, sm_count(), s);
}


// expert parallelism, source side: plan + pack the records of this rank's assignments.
int ep_dispatch(const void* x, int T, int H, const int* ids, const float* weights, int topk, int E, int G,
                int capacity, float in_gscale, const float* d_in_amax, const Workspace& w, uint8_t* records,
                int* send_counts, int* overflow, cudaStream_t s) {
    const int n_assign = T * topk;
    const int n_chunks = (n_assign + kChunk - 1) / kChunk;
    moe_hist_rank_kernel<<<n_chunks, 256, 0, s>>>(ids, n_assign, E, w.hist, w.lrank);
    ep_plan_kernel<<<1, 256, 0, s>>>(w.hist, n_chunks, E, E / G, G, capacity, w.chunk_base, w.seg_count,
                                     w.seg_start, send_counts, overflow);
    ep_pack_kernel<<<(T * kPackWarps + 7) / 8, 256, 0, s>>>(static_cast<const uint16_t*>(x), T, H, topk,
                                                            w.chunk_base, w.lrank, kChunk, E, ids, weights, E / G,
                                                            capacity, w.seg_start, in_gscale, d_in_amax, records,
                                                            w.ep_ids, EpPackPeers{});
    return launch_status();
}

// expert parallelism over peer memory, source side: as ep_dispatch, with the records stored into the destination
// ranks' receive slots and the counts + records-landed flags published by the pack kernel.
int ep_dispatch_p2p(const void* x, int T, int H, const int* ids, const float* weights, int topk, int E,
                    float in_gscale, const float* d_in_amax, const Workspace& w, const nvfp4b_ep_peers& pr,
                    int* overflow, cudaStream_t s, bool ranked = false, int chunk = kChunk) {
    const int G = pr.G, capacity = pr.capacity;
    const int n_assign = T * topk;
    const int n_chunks = (n_assign + chunk - 1) / chunk;
    if (!ranked) moe_hist_rank_kernel<<<n_chunks, 256, 0, s>>>(ids, n_assign, E, w.hist, w.lrank);
    ep_plan_kernel<<<1, 256, 0, s>>>(w.hist, n_chunks, E, E / G, G, capacity, w.chunk_base, w.seg_count,
                                     w.seg_start, w.ep_send, overflow);
    EpPackPeers pp;
    pp.recv = pr.recv;
    pp.counts = pr.counts;
    pp.flags = pr.flags;
    pp.state = pr.state;
    pp.send_counts = w.ep_send;
    pp.rank = pr.rank;
    pp.G = G;
    ep_pack_kernel<<<(T * kPackWarps + 7) / 8, 256, 0, s>>>(static_cast<const uint16_t*>(x), T, H, topk,
                                                            w.chunk_base, w.lrank, chunk, E, ids, weights, E / G,
                                                            capacity, w.seg_start, in_gscale, d_in_amax, nullptr,
                                                            w.ep_ids, pp);
    return launch_status();
}

// expert parallelism, expert side: received records -> padded expert-sorted operand -> gate/up -> down GEMM, leaving
// each record's weighted output row (fp16) in w.y in record order.
int ep_expert(const uint8_t* records, int G, int capacity, const int* recv_counts, const nvfp4b_moe_experts* ex,
              const Workspace& w, cudaStream_t s, const nvfp4b_ep_peers* peers = nullptr,
              float* zero_word = nullptr) {
    const int H = ex->hidden, E = ex->num_experts;
    const int n = G * capacity;
    const int n_chunks = (n + kChunk - 1) / kChunk;
    int* err = device_error_ptr();
    if (!err) return NVFP4B_ERR_CUDA;
    ep_meta_rank_kernel<<<n_chunks, 256, 0, s>>>(records, n, H, capacity, recv_counts, w.ep_ids, w.ep_w, E, w.hist,
                                                  w.lrank, peers ? peers->my_flags : nullptr, G,
                                                  peers ? peers->state : nullptr, err,
                                                  g_peer_wait_ns.load(std::memory_order_relaxed));
    moe_plan_kernel<<<1, kPlanThreads, 0, s>>>(w.hist, n_chunks, E, w.chunk_base, w.seg_start, w.seg_count,
                                               w.m_tiles, w.tile_expert);
    const int tile_cols = (H / 16 + 3) / 4;
    ep_scatter_kernel<<<(n + 7) / 8, 256, 0, s>>>(records, n, H, w.ep_ids, w.ep_w, E, w.chunk_base, w.lrank, w.dest,
                                                  w.row_assign, w.row_weight, w.a_codes, w.a_scales, w.row_gscale,
                                                  tile_cols);
    int st = launch_status();
    if (st) return st;
    st = gate_up<false>(ex, n, 1, 1.0f, nullptr, nullptr, w, s, true);
    if (st) return st;
    return down(ex, n, 1, w.ep_w, nullptr, 0, w, s, peers, CombineNext{nullptr, nullptr}, zero_word);
}

// Gate/up interleave: w13 row 32g + r <- gate row 16g + r; 32g + 16 + r <- up row 16g + r.
__global__ void pack_w13_kernel(const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up, int I,
                                int row_bytes, uint8_t* __restrict__ dst) {
    const int row = blockIdx.x;     // destination row
    const int g = row >> 5, r = row & 31;
    const uint8_t* src = (r < 16 ? gate : up) + (long long)(16 * g + (r & 15)) * row_bytes;
    for (int i = threadIdx.x; i < row_bytes; i += blockDim.x) dst[(long long)row * row_bytes + i] = src[i];
}

__global__ void pack_w13_scales_kernel(const uint8_t* __restrict__ gate_sf, const uint8_t* __restrict__ up_sf,
                                       int I, int kb, int tile_cols, uint8_t* __restrict__ dst, long long total) {
    for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        const long long tile = o >> 9;
        const int within = (int)(o & 511);
        const int tr = (int)(tile / tile_cols), tcol = (int)(tile % tile_cols);
        const int row = tr * 128 + ((within >> 2) & 3) * 32 + (within >> 4);
        const int b = tcol * 4 + (within & 3);
        uint8_t v = 0;
        if (row < 2 * I && b < kb) {
            const int g = row >> 5, r = row & 31;
            const uint8_t* src = r < 16 ? gate_sf : up_sf;
            v = src[(long long)(16 * g + (r & 15)) * kb + b];
        }
        dst[o] = v;
    }
}

}  // namespace
}  // namespace nvfp4b

using namespace nvfp4b;

extern "C" int nvfp4b_moe_max_rows(int T, int E, int topk) { return max_rows_for(T, E, topk); }

extern "C" size_t nvfp4b_moe_workspace_bytes(int T, int H, int I, int E, int topk) {
    if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || topk <= 0) return 0;
    return carve(nullptr, T, H, I, E, topk).bytes;
}

extern "C" int nvfp4b_moe_workspace_view(void* workspace, int T, int H, int I, int E, int topk,
                                         nvfp4b_moe_view* v) {
    if (!workspace || !v) return NVFP4B_ERR_NULL;
    const Workspace w = carve(workspace, T, H, I, E, topk);
    v->m_tiles = w.m_tiles;
    v->tile_expert = w.tile_expert;
    v->seg_start = w.seg_start;
    v->seg_count = w.seg_count;
    v->row_token = w.row_token;
    v->row_weight = w.row_weight;
    v->row_assign = w.row_assign;
    v->y = w.y;
    v->dest = w.dest;
    v->a_codes = w.a_codes;
    v->a_scales = w.a_scales;
    v->h_codes = w.h_codes;
    v->h_scales = w.h_scales;
    return NVFP4B_OK;
}

// Router launch sequence (split-K bf16 GEMM into `partial`, then softmax/top-k); arguments already checked.
// `partial` holds splits * T * E fp32 values, every one stored before it is read: nothing needs to start at zero.
// With hist/lrank (the fused MoE layer) the top-k kernel also ranks each block's chunk of 8 * tpw tokens'
// assignments for the dispatch (router_topk_rank_kernel).
static int route_launch(const void* x, int T, int H, const void* proj, int E, int topk,
                        const float* per_expert_scale, int norm, int* ids, float* weights, float* partial,
                        cudaStream_t s, int* hist = nullptr, int* lrank = nullptr) {
    CUtensorMap ma, mb;
    int st = make_kmajor_map(&ma, x, T, (long long)H * 2, RouterCfg::BM);
    if (st) return st;
    st = make_kmajor_map(&mb, proj, E, (long long)H * 2, RouterCfg::BN);
    if (st) return st;
    CoreParams cp;
    cp.err = device_error_ptr();
    if (!cp.err) return NVFP4B_ERR_CUDA;
    cp.sfa = nullptr;
    cp.sfb = nullptr;
    cp.tile_cols = (H * 2) / 32;
    cp.k_tiles = (cp.tile_cols + 3) / 4;
    SplitKSched<RouterCfg::BN> sc{};
    sc.m_tiles = (T + 127) / 128;
    sc.n_tiles = (E + RouterCfg::BN - 1) / RouterCfg::BN;
    // Enough K splits for about one tile per SM (small T has few row blocks), within router_max_splits.  Every split
    // must own at least one K tile: an empty split would store an accumulator no MMA wrote.
    const int per_split = sc.m_tiles * sc.n_tiles;
    int want = (sm_count() + per_split - 1) / per_split;
    want = want < 1 ? 1 : want > router_max_splits(T, E) ? router_max_splits(T, E) : want;
    const int kt_per_split = (cp.k_tiles + want - 1) / want;
    const int splits = (cp.k_tiles + kt_per_split - 1) / kt_per_split;
    sc.splits = splits;
    sc.kt_per_split = kt_per_split;
    sc.k_tiles = cp.k_tiles;
    sc.N = E;
    sc.b_row_tiles = (E + 127) / 128;
    RouterEpi e;
    e.partial = partial;
    e.split_stride = (long long)T * E;
    e.T = T;
    e.E = E;
    const int tiles = sc.m_tiles * sc.n_tiles * sc.splits;
    st = launch_core<RouterCfg>(ma, mb, cp, sc, e, tiles < sm_count() ? tiles : sm_count(), s);
    if (st) return st;
    const uint16_t* xn = norm ? static_cast<const uint16_t*>(x) : nullptr;
    const int epl = E / 32;
    const long long stride = (long long)T * E;
    const int tpw = router_topk_tpw(T, topk, sm_count());
    const unsigned blocks = hist ? (unsigned)((T + 8 * tpw - 1) / (8 * tpw)) : (unsigned)((T + 7) / 8);
#define NVFP4B_TOPK(EPL)                                                                                          \
    st = hist ? launch_k(router_topk_rank_kernel<EPL>, dim3(blocks), dim3(256), 0, s, (const float*)partial,       \
                         splits, stride, T, E, topk, xn, H, per_expert_scale, ids, weights, hist, lrank, tpw)     \
              : launch_k(router_topk_kernel<EPL>, dim3(blocks), dim3(256), 0, s, (const float*)partial, splits,    \
                         stride, T, E, topk, xn, H, per_expert_scale, ids, weights)
    switch (epl) {
        case 1: NVFP4B_TOPK(1); break;
        case 2: NVFP4B_TOPK(2); break;
        case 3: NVFP4B_TOPK(3); break;
        case 4: NVFP4B_TOPK(4); break;
        case 5: NVFP4B_TOPK(5); break;
        case 6: NVFP4B_TOPK(6); break;
        case 7: NVFP4B_TOPK(7); break;
        default: NVFP4B_TOPK(8); break;
    }
#undef NVFP4B_TOPK
    return st;
}

static int route_checks(const void* x, int T, int H, const void* proj, int E, int topk, const int* ids,
                        const float* weights) {
    if (!x || !proj || !ids || !weights) return NVFP4B_ERR_NULL;
    if (T <= 0 || H <= 0 || (H % 64) || E <= 0 || (E % 32) || E > 256 || topk <= 0 || topk > 16 || topk > E)
        return NVFP4B_ERR_SHAPE;
    if (!aligned16(x) || !aligned16(proj)) return NVFP4B_ERR_ALIGN;
    return NVFP4B_OK;
}

extern "C" int nvfp4b_moe_route(const void* x, int T, int H, const void* proj, int E, int topk,
                                const float* per_expert_scale, int norm, int* ids, float* weights, void* workspace,
                                void* stream) {
    if (!workspace) return NVFP4B_ERR_NULL;
    const int st = route_checks(x, T, H, proj, E, topk, ids, weights);
    if (st) return st;
    if (!aligned16(workspace)) return NVFP4B_ERR_ALIGN;
    const Workspace w = carve(workspace, T, H, 32, E, topk);   // the router part of the layout ignores I
    return route_launch(x, T, H, proj, E, topk, per_expert_scale, norm, ids, weights, w.partial,
                        (cudaStream_t)stream);
}

// ---- Router with no caller workspace and no allocation ----------------------------------------------------------
// For callers that cannot allocate or hand in scratch memory: a decode loop that reserves all of its device memory
// once, up front (the reference's decode step does exactly that, src/forward.cu:394-409, because a per-step cudaMalloc
// synchronises the device), and a host runtime whose memory planner owns every byte on the device.  Neither has a
// workspace arena to pass to nvfp4b_moe_route.  This entry keeps the split-K partial logits in a file-scope device
// array instead, so the call allocates nothing (no cudaMalloc/cudaFree, no library allocator).
//
// Limit: kRouteScratchBytes (4 MiB) of partials, i.e. router_max_splits(T, E) * T * E * 4 bytes, which holds exactly
// when T * E <= 262144 (T <= 2048 at E = 128).  Larger calls are rejected with NVFP4B_ERR_SCRATCH before anything is
// launched.
// The array is one per device and per loaded library: calls that overlap in time on the same device (two streams,
// or two host threads without ordering between their streams) race on it and produce wrong routes.
constexpr size_t kRouteScratchBytes = size_t(4) << 20;
static __device__ __align__(256) float g_route_scratch[kRouteScratchBytes / sizeof(float)];

// Device address of g_route_scratch on the current device.  The host-side symbol is not a device address, so it is
// looked up with cudaGetSymbolAddress once per device, with that device current; the first call on a device also
// loads the module there, so make it before any stream capture that should contain this entry.
static float* route_scratch_ptr() {
    static std::mutex mu;
    static float* cached[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!cached[dev]) {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_route_scratch);
        if (err != cudaSuccess) {
            record_cuda_error(err);
            return nullptr;
        }
        cached[dev] = static_cast<float*>(p);
    }
    return cached[dev];
}

extern "C" int nvfp4b_moe_route_noalloc(const void* x, int T, int H, const void* proj, int E, int topk,
                                        const float* per_expert_scale, int norm, int* ids, float* weights,
                                        void* stream) {
    const int st = route_checks(x, T, H, proj, E, topk, ids, weights);
    if (st) return st;
    if ((size_t)router_max_splits(T, E) * (size_t)T * (size_t)E * sizeof(float) > kRouteScratchBytes)
        return NVFP4B_ERR_SCRATCH;
    float* partial = route_scratch_ptr();
    if (!partial) return NVFP4B_ERR_CUDA;
    return route_launch(x, T, H, proj, E, topk, per_expert_scale, norm, ids, weights, partial, (cudaStream_t)stream);
}

static int moe_common_checks(const void* x, int T, const int* ids, const float* weights, int topk,
                             const nvfp4b_moe_experts* ex, void* workspace) {
    if (!x || !ids || !weights || !workspace) return NVFP4B_ERR_NULL;
    const int st = check_experts(ex);
    if (st) return st;
    if (T <= 0 || topk <= 0 || topk > 16 || topk > ex->num_experts) return NVFP4B_ERR_SHAPE;
    if (!aligned16(x) || !aligned16(workspace)) return NVFP4B_ERR_ALIGN;
    return NVFP4B_OK;
}

static int moe_forward(const void* x, int T, const int* ids, const float* weights, int topk,
                       const nvfp4b_moe_experts* ex, float in_gscale, const float* d_in_amax, float* out, int flags,
                       void* workspace, const CombineNext next, void* stream, const uint16_t* norm_w = nullptr,
                       float eps = 0.f) {
    int st = moe_common_checks(x, T, ids, weights, topk, ex, workspace);
    if (st) return st;
    if (!out) return NVFP4B_ERR_NULL;
    if (!aligned16(out) || (next.x && !aligned16(next.x))) return NVFP4B_ERR_ALIGN;
    if (next.x && (flags & NVFP4B_MOE_ATOMIC)) return NVFP4B_ERR_ARG;     // the chained output needs the combine
    cudaStream_t s = (cudaStream_t)stream;
    const Workspace w = carve(workspace, T, ex->hidden, ex->inter, ex->num_experts, topk);
    st = dispatch(x, T, ids, weights, topk, ex->hidden, ex->num_experts, in_gscale, d_in_amax, w, s, norm_w, eps);
    if (st) return st;
    st = gate_up<false>(ex, T, topk, in_gscale, d_in_amax, nullptr, w, s);
    if (st) return st;
    return down(ex, T, topk, weights, out, flags, w, s, nullptr, next);
}

extern "C" int nvfp4b_moe_forward(const void* x, int T, const int* ids, const float* weights, int topk,
                                  const nvfp4b_moe_experts* ex, float in_gscale, const float* d_in_amax, float* out,
                                  int flags, void* workspace, void* stream) {
    return moe_forward(x, T, ids, weights, topk, ex, in_gscale, d_in_amax, out, flags, workspace,
                       CombineNext{nullptr, nullptr}, stream);
}

extern "C" int nvfp4b_moe_forward_norm(const void* x, int T, const int* ids, const float* weights, int topk,
                                       const nvfp4b_moe_experts* ex, const void* norm_weight, float eps,
                                       float in_gscale, float* out, int flags, void* workspace, void* stream) {
    if (!norm_weight) return NVFP4B_ERR_NULL;
    if (!aligned16(norm_weight)) return NVFP4B_ERR_ALIGN;
    if (!(in_gscale > 0.0f) || !(eps >= 0.0f)) return NVFP4B_ERR_ARG;
    return moe_forward(x, T, ids, weights, topk, ex, in_gscale, nullptr, out, flags, workspace,
                       CombineNext{nullptr, nullptr}, stream, static_cast<const uint16_t*>(norm_weight), eps);
}

extern "C" int nvfp4b_moe_forward_chain(const void* x, int T, const int* ids, const float* weights, int topk,
                                        const nvfp4b_moe_experts* ex, float in_gscale, const float* d_in_amax,
                                        float* out, int flags, void* workspace, void* x_next, float* d_amax_next,
                                        void* stream) {
    if (!x_next || !d_amax_next) return NVFP4B_ERR_NULL;
    return moe_forward(x, T, ids, weights, topk, ex, in_gscale, d_in_amax, out, flags, workspace,
                       CombineNext{static_cast<uint16_t*>(x_next), d_amax_next}, stream);
}

// Router + layer in one call (the router fused into the MoE prologue): router GEMM, top-k with the dispatch ranking
// in the same kernel, plan, quantise-scatter, gate/up, down, combine -- seven launches.
extern "C" int nvfp4b_moe_layer(const void* x, int T, const void* proj, int topk, const float* per_expert_scale,
                                int norm, const nvfp4b_moe_experts* ex, float in_gscale, const float* d_in_amax,
                                float* out, int flags, int* ids, float* weights, void* workspace, void* x_next,
                                float* d_amax_next, void* stream) {
    if (!proj) return NVFP4B_ERR_NULL;
    int st = moe_common_checks(x, T, ids, weights, topk, ex, workspace);
    if (st) return st;
    const int H = ex->hidden, E = ex->num_experts;
    st = route_checks(x, T, H, proj, E, topk, ids, weights);
    if (st) return st;
    if (!out) return NVFP4B_ERR_NULL;
    if ((x_next == nullptr) != (d_amax_next == nullptr)) return NVFP4B_ERR_NULL;
    if (!aligned16(out) || (x_next && !aligned16(x_next))) return NVFP4B_ERR_ALIGN;
    if (x_next && (flags & NVFP4B_MOE_ATOMIC)) return NVFP4B_ERR_ARG;
    cudaStream_t s = (cudaStream_t)stream;
    const Workspace w = carve(workspace, T, H, ex->inter, E, topk);
    st = route_launch(x, T, H, proj, E, topk, per_expert_scale, norm, ids, weights, w.partial, s, w.hist, w.lrank);
    if (st) return st;
    st = dispatch(x, T, ids, weights, topk, H, E, in_gscale, d_in_amax, w, s, nullptr, 0.f, true,
                  8 * router_topk_tpw(T, topk, sm_count()) * topk);
    if (st) return st;
    st = gate_up<false>(ex, T, topk, in_gscale, d_in_amax, nullptr, w, s);
    if (st) return st;
    return down(ex, T, topk, weights, out, flags, w, s, nullptr,
                CombineNext{static_cast<uint16_t*>(x_next), d_amax_next});
}

extern "C" int nvfp4b_moe_dispatch(const void* x, int T, const int* ids, const float* weights, int topk,
                                   const nvfp4b_moe_experts* ex, float in_gscale, const float* d_in_amax,
                                   void* workspace, void* stream) {
    const int st = moe_common_checks(x, T, ids, weights, topk, ex, workspace);
    if (st) return st;
    const Workspace w = carve(workspace, T, ex->hidden, ex->inter, ex->num_experts, topk);
    return dispatch(x, T, ids, weights, topk, ex->hidden, ex->num_experts, in_gscale, d_in_amax, w,
                    (cudaStream_t)stream);
}

extern "C" int nvfp4b_moe_gate_up(int T, int topk, const nvfp4b_moe_experts* ex, float in_gscale,
                                  const float* d_in_amax, void* workspace, void* stream) {
    const int st = check_experts(ex);
    if (st) return st;
    if (!workspace) return NVFP4B_ERR_NULL;
    if (T <= 0 || topk <= 0 || topk > 16) return NVFP4B_ERR_SHAPE;
    const Workspace w = carve(workspace, T, ex->hidden, ex->inter, ex->num_experts, topk);
    return gate_up<false>(ex, T, topk, in_gscale, d_in_amax, nullptr, w, (cudaStream_t)stream);
}

extern "C" int nvfp4b_moe_down(int T, int topk, const float* weights, const nvfp4b_moe_experts* ex, float* out,
                               int flags, void* workspace, void* stream) {
    const int st = check_experts(ex);
    if (st) return st;
    if (!workspace || !out || !weights) return NVFP4B_ERR_NULL;
    if (!aligned16(out)) return NVFP4B_ERR_ALIGN;
    if (T <= 0 || topk <= 0 || topk > 16) return NVFP4B_ERR_SHAPE;
    const Workspace w = carve(workspace, T, ex->hidden, ex->inter, ex->num_experts, topk);
    return down(ex, T, topk, weights, out, flags, w, (cudaStream_t)stream);
}

extern "C" int nvfp4b_moe_calibrate(const void* x, int T, const int* ids, const float* weights, int topk,
                                    const nvfp4b_moe_experts* ex, float in_gscale, const float* d_in_amax,
                                    float* h_amax, void* workspace, void* stream) {
    int st = moe_common_checks(x, T, ids, weights, topk, ex, workspace);
    if (st) return st;
    if (!h_amax) return NVFP4B_ERR_NULL;
    cudaStream_t s = (cudaStream_t)stream;
    const Workspace w = carve(workspace, T, ex->hidden, ex->inter, ex->num_experts, topk);
    cudaError_t e = cudaMemsetAsync(h_amax, 0, (size_t)ex->num_experts * sizeof(float), s);
    if (e != cudaSuccess) return record_cuda_error(e);
    st = dispatch(x, T, ids, weights, topk, ex->hidden, ex->num_experts, in_gscale, d_in_amax, w, s);
    if (st) return st;
    return gate_up<true>(ex, T, topk, in_gscale, d_in_amax, h_amax, w, s);
}

extern "C" int nvfp4b_moe_pack_expert(const uint8_t* gate, const uint8_t* gate_scales, const uint8_t* up,
                                      const uint8_t* up_scales, const uint8_t* down_w, const uint8_t* down_scales,
                                      int H, int I, uint8_t* w13_dst, uint8_t* w13_scales_dst, uint8_t* w2_dst,
                                      uint8_t* w2_scales_dst, void* stream) {
    if (!gate || !gate_scales || !up || !up_scales || !down_w || !down_scales || !w13_dst || !w13_scales_dst ||
        !w2_dst || !w2_scales_dst)
        return NVFP4B_ERR_NULL;
    if (H <= 0 || I <= 0 || (H % 32) || (I % 32)) return NVFP4B_ERR_SHAPE;
    cudaStream_t s = (cudaStream_t)stream;
    pack_w13_kernel<<<2 * I, 128, 0, s>>>(gate, up, I, H / 2, w13_dst);
    const long long total = (long long)scale_bytes(2 * I, H);
    pack_w13_scales_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(gate_scales, up_scales, I, H / 16,
                                                                           (H / 16 + 3) / 4, w13_scales_dst, total);
    cudaError_t e = cudaMemcpyAsync(w2_dst, down_w, (size_t)H * (I / 2), cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return record_cuda_error(e);
    const int st = nvfp4b_swizzle_scales(down_scales, w2_scales_dst, H, I, stream);
    if (st) return st;
    return launch_status();
}

// ---- expert parallelism ------------------------------------------------------------------------------------------

extern "C" size_t nvfp4b_ep_record_bytes(int H) { return H > 0 && H % 256 == 0 ? ep_record_bytes(H) : 0; }

extern "C" int nvfp4b_ep_dispatch(const void* x, int T, int H, const int* ids, const float* weights, int topk, int E,
                                  int G, int capacity, float in_gscale, const float* d_in_amax, void* workspace,
                                  uint8_t* records, int* send_counts, int* overflow, void* stream) {
    if (!x || !ids || !weights || !workspace || !records || !send_counts || !overflow) return NVFP4B_ERR_NULL;
    if (T <= 0 || H <= 0 || (H % 256) || topk <= 0 || topk > 16 || E <= 0 || E > 256 || G <= 0 || G > 256 ||
        (E % G) || topk > E || capacity <= 0)
        return NVFP4B_ERR_SHAPE;
    if (!aligned16(x) || !aligned16(records) || !aligned16(workspace)) return NVFP4B_ERR_ALIGN;
    const Workspace w = carve(workspace, T, H, 32, E, topk);
    return ep_dispatch(x, T, H, ids, weights, topk, E, G, capacity, in_gscale, d_in_amax, w, records, send_counts,
                       overflow, (cudaStream_t)stream);
}

extern "C" int nvfp4b_ep_expert_forward(const uint8_t* records, int G, int capacity, const int* recv_counts,
                                        const nvfp4b_moe_experts* ex, void* workspace, void* stream) {
    if (!records || !recv_counts || !workspace) return NVFP4B_ERR_NULL;
    const int st = check_experts(ex);
    if (st) return st;
    if (G <= 0 || capacity <= 0 || (long long)G * capacity > (1 << 26)) return NVFP4B_ERR_SHAPE;
    if (!aligned16(records) || !aligned16(workspace)) return NVFP4B_ERR_ALIGN;
    const Workspace w = carve(workspace, G * capacity, ex->hidden, ex->inter, ex->num_experts, 1);
    return ep_expert(records, G, capacity, recv_counts, ex, w, (cudaStream_t)stream);
}

extern "C" int nvfp4b_ep_combine(const uint16_t* y_back, int T, int H, int topk, int E, const void* workspace,
                                 float* out, int flags, void* stream) {
    if (!y_back || !workspace || !out) return NVFP4B_ERR_NULL;
    if (T <= 0 || H <= 0 || (H % 256) || topk <= 0 || topk > 16 || E <= 0) return NVFP4B_ERR_SHAPE;
    if (flags & ~NVFP4B_MOE_ACCUMULATE) return NVFP4B_ERR_ARG;
    if (!aligned16(y_back) || !aligned16(out)) return NVFP4B_ERR_ALIGN;
    const Workspace w = carve(const_cast<void*>(workspace), T, H, 32, E, topk);
    const long long threads = (long long)T * (H / 8);
    ep_combine_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        y_back, T, H, topk, w.ep_ids, out, (flags & NVFP4B_MOE_ACCUMULATE) ? 1 : 0, nullptr, 0, nullptr, nullptr, 0ull,
        CombineNext{nullptr, nullptr});
    return launch_status();
}

// ---- expert parallelism over peer memory ---------------------------------------------------------------------

static int check_peers(const nvfp4b_ep_peers* p) {
    if (!p || !p->recv || !p->back || !p->counts || !p->flags || !p->my_recv || !p->my_back || !p->my_counts ||
        !p->my_flags || !p->state)
        return NVFP4B_ERR_NULL;
    if (p->G <= 0 || p->G > 256 || p->rank < 0 || p->rank >= p->G || p->capacity <= 0 ||
        (long long)p->G * p->capacity > (1 << 26))
        return NVFP4B_ERR_SHAPE;
    if (!aligned16(p->my_recv) || !aligned16(p->my_back)) return NVFP4B_ERR_ALIGN;
    return NVFP4B_OK;
}

static size_t p2p_layout(int G, int capacity, int H, size_t* off) {
    const size_t n = (size_t)G * capacity;
    size_t o[5];
    o[0] = 0;
    o[1] = o[0] + align256(n * ep_record_bytes(H));
    o[2] = o[1] + align256(n * (size_t)H * 2);
    o[3] = o[2] + align256((size_t)G * 4);
    o[4] = o[3] + align256((size_t)2 * G * 4);
    if (off)
        for (int i = 0; i < 5; ++i) off[i] = o[i];
    return o[4] + 256;
}

extern "C" size_t nvfp4b_ep_p2p_buffer_bytes(int G, int capacity, int H, size_t* offsets) {
    if (G <= 0 || G > 256 || capacity <= 0 || H <= 0 || (H % 256)) return 0;
    return p2p_layout(G, capacity, H, offsets);
}

extern "C" int nvfp4b_ep_p2p_dispatch(const void* x, int T, int H, const int* ids, const float* weights, int topk,
                                      int E, float in_gscale, const float* d_in_amax, void* workspace,
                                      const nvfp4b_ep_peers* peers, int* overflow, void* stream) {
    if (!x || !ids || !weights || !workspace || !overflow) return NVFP4B_ERR_NULL;
    const int st = check_peers(peers);
    if (st) return st;
    const int G = peers->G;
    if (T <= 0 || H <= 0 || (H % 256) || topk <= 0 || topk > 16 || E <= 0 || E > 256 || (E % G) || topk > E)
        return NVFP4B_ERR_SHAPE;
    if (!aligned16(x) || !aligned16(workspace)) return NVFP4B_ERR_ALIGN;
    const Workspace w = carve(workspace, T, H, 32, E, topk);
    return ep_dispatch_p2p(x, T, H, ids, weights, topk, E, in_gscale, d_in_amax, w, *peers, overflow,
                           (cudaStream_t)stream);
}

extern "C" int nvfp4b_ep_p2p_expert_forward(const nvfp4b_moe_experts* ex, void* workspace,
                                            const nvfp4b_ep_peers* peers, void* stream) {
    if (!workspace) return NVFP4B_ERR_NULL;
    int st = check_experts(ex);
    if (st) return st;
    st = check_peers(peers);
    if (st) return st;
    if (!aligned16(workspace)) return NVFP4B_ERR_ALIGN;
    const int n = peers->G * peers->capacity;
    const Workspace w = carve(workspace, n, ex->hidden, ex->inter, ex->num_experts, 1);
    return ep_expert(peers->my_recv, peers->G, peers->capacity, peers->my_counts, ex, w, (cudaStream_t)stream,
                     peers);
}

static int ep_p2p_combine(int T, int H, int topk, int E, const void* workspace, const nvfp4b_ep_peers* peers,
                          float* out, int flags, const CombineNext next, void* stream, bool amax_zeroed = false) {
    if (!workspace || !out) return NVFP4B_ERR_NULL;
    const int st = check_peers(peers);
    if (st) return st;
    if (T <= 0 || H <= 0 || (H % 256) || topk <= 0 || topk > 16 || E <= 0) return NVFP4B_ERR_SHAPE;
    if (flags & ~NVFP4B_MOE_ACCUMULATE) return NVFP4B_ERR_ARG;
    if (!aligned16(out) || (next.x && !aligned16(next.x))) return NVFP4B_ERR_ALIGN;
    int* err = device_error_ptr();
    if (!err) return NVFP4B_ERR_CUDA;
    const cudaStream_t s = (cudaStream_t)stream;
    if (next.x && !amax_zeroed) {
        const cudaError_t e = cudaMemsetAsync(next.amax, 0, sizeof(float), s);
        if (e != cudaSuccess) return record_cuda_error(e);
    }
    const Workspace w = carve(const_cast<void*>(workspace), T, H, 32, E, topk);
    const long long threads = (long long)T * (H / 8);
    ep_combine_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
        peers->my_back, T, H, topk, w.ep_ids, out, (flags & NVFP4B_MOE_ACCUMULATE) ? 1 : 0, peers->my_flags + peers->G,
        peers->G, peers->state, err, g_peer_wait_ns.load(std::memory_order_relaxed), next);
    return launch_status();
}

extern "C" int nvfp4b_ep_p2p_combine(int T, int H, int topk, int E, const void* workspace,
                                     const nvfp4b_ep_peers* peers, float* out, int flags, void* stream) {
    return ep_p2p_combine(T, H, topk, E, workspace, peers, out, flags, CombineNext{nullptr, nullptr}, stream);
}

extern "C" int nvfp4b_ep_p2p_combine_chain(int T, int H, int topk, int E, const void* workspace,
                                           const nvfp4b_ep_peers* peers, float* out, int flags, void* x_next,
                                           float* d_amax_next, void* stream) {
    if (!x_next || !d_amax_next) return NVFP4B_ERR_NULL;
    return ep_p2p_combine(T, H, topk, E, workspace, peers, out, flags,
                          CombineNext{static_cast<uint16_t*>(x_next), d_amax_next}, stream);
}

// Router + one expert-parallel layer on this rank in one call: the router top-k shares its kernel with the
// dispatch ranking, the chained amax is reset inside the down GEMM (no memset).
extern "C" int nvfp4b_ep_p2p_layer(const void* x, int T, const void* proj, int topk, const float* per_expert_scale,
                                   int norm, int E, const nvfp4b_moe_experts* local_experts, float in_gscale,
                                   const float* d_in_amax, float* out, int flags, int* ids, float* weights,
                                   void* src_workspace, void* exp_workspace, const nvfp4b_ep_peers* peers,
                                   int* overflow, void* x_next, float* d_amax_next, void* stream) {
    if (!x || !proj || !ids || !weights || !src_workspace || !exp_workspace || !overflow || !out)
        return NVFP4B_ERR_NULL;
    if ((x_next == nullptr) != (d_amax_next == nullptr)) return NVFP4B_ERR_NULL;
    int st = check_experts(local_experts);
    if (st) return st;
    st = check_peers(peers);
    if (st) return st;
    const int G = peers->G, H = local_experts->hidden;
    if (local_experts->num_experts * G != E) return NVFP4B_ERR_SHAPE;
    st = route_checks(x, T, H, proj, E, topk, ids, weights);
    if (st) return st;
    if (flags & ~NVFP4B_MOE_ACCUMULATE) return NVFP4B_ERR_ARG;
    if (!aligned16(src_workspace) || !aligned16(exp_workspace) || !aligned16(out) || (x_next && !aligned16(x_next)))
        return NVFP4B_ERR_ALIGN;
    const cudaStream_t s = (cudaStream_t)stream;
    const Workspace ws = carve(src_workspace, T, H, 32, E, topk);
    st = route_launch(x, T, H, proj, E, topk, per_expert_scale, norm, ids, weights, ws.partial, s, ws.hist, ws.lrank);
    if (st) return st;
    st = ep_dispatch_p2p(x, T, H, ids, weights, topk, E, in_gscale, d_in_amax, ws, *peers, overflow, s, true,
                         8 * router_topk_tpw(T, topk, sm_count()) * topk);
    if (st) return st;
    const Workspace we = carve(exp_workspace, G * peers->capacity, H, local_experts->inter,
                               local_experts->num_experts, 1);
    // the pack kernel above was the last reader of this layer's input scale on this rank
    st = ep_expert(peers->my_recv, G, peers->capacity, peers->my_counts, local_experts, we, s, peers, d_amax_next);
    if (st) return st;
    return ep_p2p_combine(T, H, topk, E, src_workspace, peers, out, flags,
                          CombineNext{static_cast<uint16_t*>(x_next), d_amax_next}, stream, true);
}

extern "C" int nvfp4b_ep_set_peer_wait_ns(unsigned long long ns) {
    if (ns == 0) ns = kPeerWaitDefaultNs;
    if (ns < 1000ull || ns > 600000000000ull) return NVFP4B_ERR_ARG;
    g_peer_wait_ns.store(ns, std::memory_order_relaxed);
    return NVFP4B_OK;
}

extern "C" int nvfp4b_ep_p2p_state(const nvfp4b_ep_peers* peers, unsigned* host_words4) {
    if (!peers || !peers->state || !host_words4) return NVFP4B_ERR_NULL;
    const cudaError_t e = cudaMemcpy(host_words4, peers->state, 4 * sizeof(unsigned), cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? NVFP4B_OK : record_cuda_error(e);
}

extern "C" int nvfp4b_ep_p2p_recv_counts(const nvfp4b_ep_peers* peers, int* host_counts) {
    if (!peers || !peers->my_counts || !host_counts) return NVFP4B_ERR_NULL;
    if (peers->G <= 0 || peers->G > 256) return NVFP4B_ERR_SHAPE;
    const cudaError_t e = cudaMemcpy(host_counts, peers->my_counts, peers->G * sizeof(int), cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? NVFP4B_OK : record_cuda_error(e);
}

extern "C" int nvfp4b_ipc_alloc(size_t bytes, void** ptr) {
    if (!ptr) return NVFP4B_ERR_NULL;
    if (bytes == 0) return NVFP4B_ERR_SHAPE;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) return record_cuda_error(e);
    e = cudaMemset(*ptr, 0, bytes);
    if (e != cudaSuccess) return record_cuda_error(e);
    return NVFP4B_OK;
}

extern "C" int nvfp4b_ipc_free(void* ptr) {
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? NVFP4B_OK : record_cuda_error(e);
}

extern "C" int nvfp4b_ipc_handle(void* ptr, void* handle64) {
    if (!ptr || !handle64) return NVFP4B_ERR_NULL;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    const cudaError_t e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle64), ptr);
    return e == cudaSuccess ? NVFP4B_OK : record_cuda_error(e);
}

extern "C" int nvfp4b_ipc_open(const void* handle64, void** ptr) {
    if (!handle64 || !ptr) return NVFP4B_ERR_NULL;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? NVFP4B_OK : record_cuda_error(e);
}

extern "C" int nvfp4b_ipc_close(void* ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? NVFP4B_OK : record_cuda_error(e);
}
