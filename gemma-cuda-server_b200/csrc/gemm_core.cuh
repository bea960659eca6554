// gemm_core.cuh -- the NVFP4 tcgen05 GEMM kernel template shared by the dense GEMM and the MoE grouped GEMMs.
//
// D = A[rows, K] @ B[cols, K]^T, A and B packed e2m1 (K-major) with e4m3 block scales in the 128x4-tile layout,
// fp32 accumulation in TMEM (tcgen05.mma kind::mxf4nvf4, scale_vec::4X).  One CTA per SM, persistent over output
// tiles of 128 x BN:
//   warp 0            TMA producer.  Per K-tile (256 values = 128 bytes per row): one 2-D tensor load of A
//                     (128 rows) and of B (BN rows), both 128-byte swizzled, plus 1-D bulk loads of the scale tiles
//                     (the tile layout puts the scales of 128 rows x 256 K into 2 KB of contiguous memory).
//   warp 1            TMEM owner and MMA issuer (one elected thread): four 128 x N x 64 MMAs per K-tile reading
//                     their scales from the TMEM scale slot of the stage; tcgen05.commit releases the smem stage, and
//                     a commit per output tile hands the accumulator to the epilogue.
//   warps 2, 3        scale copiers: tcgen05.cp 32x128b.warpx4 moves each 512-byte scale tile (32 rows x 16 bytes)
//                     into 4 TMEM columns, replicated over the four lane quadrants as the MMA reads them.  The copies
//                     are issued apart from the MMAs, split over two threads, into one TMEM slot per smem stage:
//                     a tcgen05.cp costs the tensor pipe tens of cycles, and issued in line with the MMAs the 12
//                     copies of a 128 x 256 K-tile nearly doubled its time.
//   warps 4..         epilogue (EPI_WARPS warps): warp w reads TMEM lane quadrant w % 4; with 8 warps each quadrant
//                     is split into two column halves.  Each thread drains its 32-column chunks to registers,
//                     releases the accumulator (so the next tile's MMAs start), then runs the epilogue policy.
// Scheduler policies map a linear tile index to (A row block, B row block, expert); epilogue policies consume the
// accumulator rows.  Every wait is bounded (sm100::mbar_wait): a stuck pipeline records an error and exits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "sm100.cuh"

namespace nvfp4b {

// Operand kinds: NVF4 = e2m1 codes with e4m3 block scales (kind::mxf4nvf4, K = 64 per MMA); BF16 = plain bf16
// (kind::f16, K = 16 per MMA, no scales).  Either way one MMA consumes 32 bytes of each operand row, so a K-tile
// of 128 bytes is four MMAs and the shared-memory descriptors advance by 32 bytes per MMA.
enum class Kind { NVF4, BF16 };

// TMEM scale slots: one per smem stage.  The copier warps fill slot s from stage s as soon as the stage's loads
// land, so they run ahead of the MMAs by up to STAGES - 1 K-tiles; a slot is free again when its stage is (the
// producer refills stage s only after the MMAs that read slot s completed), so no separate release is needed.
template <int BN_, int STAGES_, int ACC_BUFS_, int EPI_WARPS_, Kind KIND_ = Kind::NVF4, int EPI_SMEM_ = 0>
struct KCfg {
    static constexpr int EPI_SMEM = EPI_SMEM_;           // extra shared memory handed to the epilogue policy
    static constexpr int BM = 128, BN = BN_, STAGES = STAGES_, ACC_BUFS = ACC_BUFS_, EPI_WARPS = EPI_WARPS_;
    static constexpr Kind KIND = KIND_;
    static constexpr bool SCALED = KIND_ == Kind::NVF4;
    static constexpr int THREADS = 128 + 32 * EPI_WARPS;  // warps 0-3 control, 4.. epilogue
    static constexpr int KT_BYTES = 128;                 // one K-tile = 128 bytes per row (256 e2m1 or 64 bf16)
    static constexpr int A_BYTES = BM * KT_BYTES;        // 16 KB
    static constexpr int B_BYTES = BN * KT_BYTES;
    static constexpr int SFA_BYTES = SCALED ? 4 * 512 : 0;   // 4 K-steps of 64 x one 128-row scale tile
    static constexpr int SFB_TILES = BN / 128;
    static constexpr int SFB_BYTES = SCALED ? SFB_TILES * 4 * 512 : 0;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
    static constexpr int SF_COLS_A = SCALED ? 16 : 0, SF_COLS_B = SCALED ? 4 * (BN / 32) : 0;
    static constexpr int SF_COL0 = ACC_BUFS * BN;
    static constexpr int TMEM_COLS = 512;
    static constexpr int SF_SLOTS = STAGES;
    static constexpr int COLS_PER_WARP = BN * 4 / EPI_WARPS;
    static constexpr int CHUNKS = COLS_PER_WARP / 32;
    static constexpr int BAR_BYTES = ((3 * STAGES + 2 * ACC_BUFS) * 8 + 16 + 127) / 128 * 128;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + EPI_SMEM + 1024;
    static_assert(SF_COL0 + SF_SLOTS * (SF_COLS_A + SF_COLS_B) <= TMEM_COLS, "TMEM budget");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(BN % 128 == 0 && BN <= 256, "BN");
    static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
    static_assert(COLS_PER_WARP % 32 == 0, "chunking");
};

// What the producer and MMA issuer need for one output tile.
struct TileInfo {
    int a_row;         // first A row (128-row block, also the A scale tile row)
    int b_row;         // first B row in the B tensor map (includes the expert offset)
    int sfb_tile0;     // first 128-row scale tile of B (includes the expert offset)
    int sfb_tiles;     // how many of the tile's 128-row B scale tiles exist (the rest are skipped)
    int n0;            // first output column (within the expert)
    int expert;        // expert id (0 for dense)
    int mb;            // 128-row block index
    int n_mma;         // MMA N for this tile (BN, or 128 for a half-empty last tile)
    int kt0, kt1;      // K-tile range [kt0, kt1) (split-K schedules; otherwise the whole K)
    int split;         // split-K index (0 otherwise)
};

struct CoreParams {
    int* err;          // device error word (runtime.cu), written when a bounded wait expires
    const uint8_t* sfa;
    const uint8_t* sfb;
    int tile_cols;     // number of 32-byte MMA K-steps along K (NVF4: = scale tiles along K = ceil(K/64))
    int k_tiles;       // 128-byte K-tiles
};

// ---------------------------------------------------------------------------------------------------------------
// Scheduler policies
// ---------------------------------------------------------------------------------------------------------------

// Grouped rasterisation: groups of `group_m` row blocks, column blocks iterated inside a group, so concurrently
// running CTAs share a few A row blocks and a few B column blocks in L2.
__device__ __forceinline__ void raster(int t, int m_tiles, int n_tiles, int group_m, int& mb, int& nb) {
    const int per_group = group_m * n_tiles;
    const int g = t / per_group;
    const int first_m = g * group_m;
    const int gsize = min(group_m, m_tiles - first_m);
    const int local = t - g * per_group;
    mb = first_m + local % gsize;
    nb = local / gsize;
}

template <int BN>
struct DenseSched {
    int m_tiles, n_tiles, group_m, N, b_row_tiles;
    __device__ __forceinline__ int num_tiles() const { return m_tiles * n_tiles; }
    __device__ __forceinline__ TileInfo tile(int t) const {
        TileInfo ti;
        int mb, nb;
        raster(t, m_tiles, n_tiles, group_m, mb, nb);
        ti.mb = mb;
        ti.a_row = mb * 128;
        ti.n0 = nb * BN;
        ti.b_row = ti.n0;
        ti.sfb_tile0 = nb * (BN / 128);
        ti.sfb_tiles = min(BN / 128, b_row_tiles - ti.sfb_tile0);
        ti.expert = 0;
        ti.n_mma = (BN > 128 && N - ti.n0 <= 128) ? 128 : BN;
        ti.kt0 = 0;
        ti.kt1 = k_tiles;
        ti.split = 0;
        return ti;
    }
    int k_tiles;
};

// Split-K over a dense problem: tile t = (split, mb, nb) with split slowest; split s covers K-tiles
// [s * kt_per_split, min((s+1) * kt_per_split, k_tiles)).
template <int BN>
struct SplitKSched {
    int m_tiles, n_tiles, splits, kt_per_split, k_tiles, N, b_row_tiles;
    __device__ __forceinline__ int num_tiles() const { return m_tiles * n_tiles * splits; }
    __device__ __forceinline__ TileInfo tile(int t) const {
        TileInfo ti;
        const int per_split = m_tiles * n_tiles;
        ti.split = t / per_split;
        const int r = t - ti.split * per_split;
        const int mb = r % m_tiles, nb = r / m_tiles;
        ti.mb = mb;
        ti.a_row = mb * 128;
        ti.n0 = nb * BN;
        ti.b_row = ti.n0;
        ti.sfb_tile0 = nb * (BN / 128);
        ti.sfb_tiles = min(BN / 128, b_row_tiles - ti.sfb_tile0);
        ti.expert = 0;
        ti.n_mma = (BN > 128 && N - ti.n0 <= 128) ? 128 : BN;
        ti.kt0 = ti.split * kt_per_split;
        ti.kt1 = min(ti.kt0 + kt_per_split, k_tiles);
        return ti;
    }
};

// MoE: A = expert-sorted rows, every expert segment padded to a multiple of 128 rows; tile_expert[mb] names the
// expert of row block mb; *d_m_tiles is the number of row blocks (written by the dispatch kernel).  B holds all
// experts' matrices stacked: rows [e * n_per_expert, (e+1) * n_per_expert).
template <int BN>
struct GroupedSched {
    const int* d_m_tiles;
    const int* tile_expert;
    int n_tiles, group_m, n_per_expert, b_row_tiles_per_expert, k_tiles;
    int m_tiles_cached;
    __device__ __forceinline__ void init() { m_tiles_cached = *(volatile const int*)d_m_tiles; }
    __device__ __forceinline__ int num_tiles() const { return m_tiles_cached * n_tiles; }
    __device__ __forceinline__ TileInfo tile(int t) const {
        TileInfo ti;
        int mb, nb;
        raster(t, m_tiles_cached, n_tiles, group_m, mb, nb);
        const int e = __ldg(tile_expert + mb);
        ti.mb = mb;
        ti.expert = e;
        ti.a_row = mb * 128;
        ti.n0 = nb * BN;
        ti.b_row = e * n_per_expert + ti.n0;
        const int rt = nb * (BN / 128);
        ti.sfb_tile0 = e * b_row_tiles_per_expert + rt;
        ti.sfb_tiles = min(BN / 128, b_row_tiles_per_expert - rt);
        ti.n_mma = (BN > 128 && n_per_expert - ti.n0 <= 128) ? 128 : BN;
        ti.kt0 = 0;
        ti.kt1 = k_tiles;
        ti.split = 0;
        return ti;
    }
};

template <class S>
__device__ __forceinline__ void sched_init(S& s) {}
template <int BN>
__device__ __forceinline__ void sched_init(GroupedSched<BN>& s) { s.init(); }

// Scale copies of one K-tile, split between the two copier warps.  BN = 256: warp p copies B scale tile p for every
// K-step and the A tile of the K-steps j with j % 2 == p (6 + 6 copies); BN = 128: warp 0 copies A, warp 1 B.  Each
// warp then reads one 2 KB run of shared memory per B tile and writes its own TMEM columns; this split measured
// about 20% faster than dealing the copies out one by one.
template <class C, bool PAIR>
__device__ __forceinline__ void issue_scale_copies(int part, int nks, uint32_t sfa_col, uint32_t sfb_col,
                                                   uint32_t sfa_base, uint32_t sfb_base) {
    using namespace sm100;
    for (int j = 0; j < nks; ++j) {
        const bool do_a = C::BN == 256 ? (j & 1) == part : part == 0;
        const bool do_b = C::BN == 256 || part == 1;
        const int h = C::BN == 256 ? part : 0;
        if (do_a) {
            if constexpr (PAIR) tmem_cp_32x128b_x4_pair(sfa_col + 4 * j, desc_sf_32x16(sfa_base + j * 512));
            else tmem_cp_32x128b_x4(sfa_col + 4 * j, desc_sf_32x16(sfa_base + j * 512));
        }
        if (do_b) {
            const uint32_t col = sfb_col + (C::BN / 32) * j + 4 * h;
            const uint64_t d = desc_sf_32x16(sfb_base + h * 2048 + j * 512);
            if constexpr (PAIR) tmem_cp_32x128b_x4_pair(col, d);
            else tmem_cp_32x128b_x4(col, d);
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------------------------------------------

template <class C, class Sched, class Epi>
__global__ void __launch_bounds__(C::THREADS, 1)
    nvf4_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const CoreParams cp, Sched sched, const Epi epi) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + C::STAGES * C::A_BYTES;
    uint8_t* sSFA = sB + C::STAGES * C::B_BYTES;
    uint8_t* sSFB = sSFA + C::STAGES * C::SFA_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + C::STAGES * C::SFB_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + C::ACC_BUFS;
    uint64_t* sf_full = tempty + C::ACC_BUFS;     // per stage: its scales are in TMEM slot `stage`
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sf_full + C::STAGES);
    volatile int* sflag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* esm = sSFB + C::STAGES * C::SFB_BYTES + C::BAR_BYTES;   // 128-byte aligned epilogue scratch

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < C::ACC_BUFS; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 32 * C::EPI_WARPS); }
        for (int b = 0; b < C::STAGES; ++b) mbar_init(&sf_full[b], 2);
        *sflag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tma_a); prefetch_tmap(&tma_b); }
    if (warp == 1) { tmem_alloc(tmem_slot, C::TMEM_COLS); tmem_relinquish(); }
    sched_init(sched);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int num_tiles = sched.num_tiles();

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const TileInfo ti = sched.tile(t);
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, sflag, kErrTimeoutProducer)) { ok = false; break; }
                    const int ks0 = kt * 4;
                    const int nks = min(4, cp.tile_cols - ks0);
                    const uint32_t sf_bytes = C::SCALED ? (uint32_t)nks * 512u : 0u;
                    mbar_arrive_expect_tx(&full[stage], (uint32_t)(C::A_BYTES + C::B_BYTES) +
                                                            sf_bytes * (1u + (uint32_t)ti.sfb_tiles));
                    tma_load_2d(sA + stage * C::A_BYTES, &tma_a, &full[stage], kt * C::KT_BYTES, ti.a_row);
                    tma_load_2d(sB + stage * C::B_BYTES, &tma_b, &full[stage], kt * C::KT_BYTES, ti.b_row);
                    if constexpr (C::SCALED) {
                        bulk_load(sSFA + stage * C::SFA_BYTES,
                                  cp.sfa + ((long long)ti.mb * cp.tile_cols + ks0) * 512, sf_bytes, &full[stage]);
                        for (int h = 0; h < ti.sfb_tiles; ++h)
                            bulk_load(sSFB + stage * C::SFB_BYTES + h * 2048,
                                      cp.sfb + ((long long)(ti.sfb_tile0 + h) * cp.tile_cols + ks0) * 512, sf_bytes,
                                      &full[stage]);
                    }
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int stage = 0, abuf = 0;
            uint32_t phase = 0, aphase = 0;
            bool ok = true;
            const uint32_t sfa_col = tmem + (uint32_t)C::SF_COL0;
            const uint32_t sfb_col = sfa_col + C::SF_COLS_A;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const TileInfo ti = sched.tile(t);
                const uint32_t idesc = C::SCALED ? idesc_nvf4(C::BM, ti.n_mma) : idesc_bf16(C::BM, ti.n_mma);
                if (!mbar_wait(&tempty[abuf], aphase ^ 1u, sflag, kErrTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(abuf * C::BN);
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!mbar_wait(&full[stage], phase, sflag, kErrTimeoutMma)) { ok = false; break; }
                    tc_fence_after();
                    const int nks = min(4, cp.tile_cols - kt * 4);
                    const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
                    const uint32_t sfa_base = smem_u32(sSFA + stage * C::SFA_BYTES);
                    const uint32_t sfb_base = smem_u32(sSFB + stage * C::SFB_BYTES);
                    const uint32_t acc0 = kt != ti.kt0 ? 1u : 0u;
                    if constexpr (C::SCALED) {
                        if (!mbar_wait(&sf_full[stage], phase, sflag, kErrTimeoutMma)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t so = (uint32_t)(stage * (C::SF_COLS_A + C::SF_COLS_B));
                        for (int j = 0; j < nks; ++j)
                            mma_nvf4(d_tmem, desc_kmajor_sw128(a_base + 32 * j), desc_kmajor_sw128(b_base + 32 * j),
                                     idesc, sfa_col + so + 4 * j, sfb_col + so + (C::BN / 32) * j,
                                     (acc0 | j) != 0 ? 1u : 0u);
                    } else {
                        for (int j = 0; j < nks; ++j)
                            mma_bf16(d_tmem, desc_kmajor_sw128(a_base + 32 * j), desc_kmajor_sw128(b_base + 32 * j),
                                     idesc, (acc0 | j) != 0 ? 1u : 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit(&tfull[abuf]);
                if (++abuf == C::ACC_BUFS) { abuf = 0; aphase ^= 1u; }
            }
        }
    } else if (warp < 4) {
        // ---------------- scale copier (warps 2, 3) ----------------
        if (C::SCALED && lane == 0) {
            const int part = warp - 2;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            const uint32_t sfa_col = tmem + (uint32_t)C::SF_COL0;
            const uint32_t sfb_col = sfa_col + C::SF_COLS_A;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const TileInfo ti = sched.tile(t);
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!mbar_wait(&full[stage], phase, sflag, kErrTimeoutMma)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t so = (uint32_t)(stage * (C::SF_COLS_A + C::SF_COLS_B));
                    issue_scale_copies<C, false>(part, min(4, cp.tile_cols - kt * 4), sfa_col + so, sfb_col + so,
                                                 smem_u32(sSFA + stage * C::SFA_BYTES),
                                                 smem_u32(sSFB + stage * C::SFB_BYTES));
                    tc_commit(&sf_full[stage]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int ew = warp - 4;
        const int quad = warp & 3;
        const int col_base = (ew >> 2) * C::COLS_PER_WARP;   // 0 with 4 warps; 0 / BN/2 with 8 warps
        const int row = quad * 32 + lane;
        int abuf = 0;
        uint32_t aphase = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            const TileInfo ti = sched.tile(t);
            // a warp whose 32 rows the epilogue policy marks dead (padding) neither loads nor processes them; the
            // policy's row lookup is made before the wait so its latency stays off the accumulator hand-off
            const bool work = col_base < ti.n_mma && __any_sync(0xFFFFFFFFu, epi.row_live(ti, row));
            if (!mbar_wait(&tfull[abuf], aphase, sflag, kErrTimeoutEpilogue)) break;
            tc_fence_after();
            const uint32_t addr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(abuf * C::BN + col_base);
            uint32_t r[C::CHUNKS][32];
            if (work) {
#pragma unroll
                for (int c = 0; c < C::CHUNKS; ++c) tmem_ld_32x32b_x32(addr + 32 * c, r[c]);
                tmem_wait_ld();
            }
            tc_fence_before();
            mbar_arrive(&tempty[abuf]);          // accumulator drained: the next tile's MMAs may start
            if (work) epi.template process<C::CHUNKS>(ti, row, col_base, r, esm);
            if (++abuf == C::ACC_BUFS) { abuf = 0; aphase ^= 1u; }
        }
        epi.finish();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
    if (threadIdx.x == 0 && *sflag != 0) atomicCAS(cp.err, 0, *sflag);
}

// ---------------------------------------------------------------------------------------------------------------
// CTA-pair kernel (tcgen05 cta_group::2)
// ---------------------------------------------------------------------------------------------------------------
// A cluster of two CTAs, one per SM of a TPC, computes a 256 x 256 output tile with M = 256 MMAs issued by the
// leader (cluster rank 0).  Each CTA stages its own 128 A rows and half of the 256 B rows, so one K-tile costs each
// SM 32 KB of operand traffic instead of 48 KB for a 128 x 256 tile, and each scale copy instruction now serves
// twice the MMA work (the copies, not the MMAs, bound the single-CTA kernel).  Each CTA's TMEM holds its 128
// accumulator rows and the scales for them (A: own rows; B: all 256 columns, staged in both CTAs).
//   warp 0 (both)     producer: A, B, scale loads of its CTA, completion counted on the LEADER's full barrier
//                     (tensor loads with cta_group::2; the leader posts the byte count of both CTAs).
//   warp 1 (leader)   MMAs for the pair; commits release the stage in both CTAs and hand the accumulator to both
//                     CTAs' epilogues.  (warp 1 of the peer only allocates TMEM.)
//   warps 2-3 (leader) scale copies for the pair (cta_group::2), into one TMEM scale slot per smem stage.
//   warps 4.. (both)  epilogue of the CTA's 128 rows; one arrival per warp on the leader's accumulator-empty barrier.
template <int STAGES_, int EPI_WARPS_, int EPI_SMEM_ = 0>
struct PairCfg {
    static constexpr int EPI_SMEM = EPI_SMEM_;
    static constexpr int BM = 128, PAIR_M = 256, BN = 256, STAGES = STAGES_, ACC_BUFS = 1, EPI_WARPS = EPI_WARPS_;
    static constexpr bool SCALED = true;
    static constexpr int THREADS = 128 + 32 * EPI_WARPS;     // warps 0-3 control, 4.. epilogue
    static constexpr int KT_BYTES = 128;
    static constexpr int A_BYTES = BM * KT_BYTES;             // 16 KB: this CTA's 128 rows
    static constexpr int B_BYTES = (BN / 2) * KT_BYTES;       // 16 KB: this CTA's half of the 256 B rows
    static constexpr int SFA_BYTES = 4 * 512;                 // one 128-row scale tile, 4 K-steps
    static constexpr int SFB_BYTES = 2 * 4 * 512;             // both 128-row scale tiles of B
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
    static constexpr uint32_t PAIR_TX = 2u * STAGE_BYTES;     // bytes the leader's full barrier waits for
    static constexpr int SF_COLS_A = 16, SF_COLS_B = 32, SF_COL0 = BN;
    static constexpr int TMEM_COLS = 512;
    static constexpr int SF_SLOTS = STAGES;
    static constexpr int COLS_PER_WARP = BN * 4 / EPI_WARPS;
    static constexpr int CHUNKS = COLS_PER_WARP / 32;
    static constexpr int BAR_BYTES = ((3 * STAGES + 2) * 8 + 16 + 127) / 128 * 128;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + EPI_SMEM + 1024;
    static_assert(SF_COL0 + SF_SLOTS * (SF_COLS_A + SF_COLS_B) <= TMEM_COLS, "TMEM budget");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
};

// Dense problem in 256 x 256 pair tiles; TileInfo describes the pair (a_row = first of 256 rows, mb = 256-row
// block); each CTA adds rank * 128 for its own rows.
struct PairDenseSched {
    int m_tiles, n_tiles, group_m, k_tiles;
    __device__ __forceinline__ int num_tiles() const { return m_tiles * n_tiles; }
    __device__ __forceinline__ TileInfo tile(int t) const {
        TileInfo ti;
        int mb, nb;
        raster(t, m_tiles, n_tiles, group_m, mb, nb);
        ti.mb = mb;
        ti.a_row = mb * 256;
        ti.n0 = nb * 256;
        ti.b_row = ti.n0;
        ti.sfb_tile0 = nb * 2;
        ti.sfb_tiles = 2;
        ti.expert = 0;
        ti.n_mma = 256;
        ti.kt0 = 0;
        ti.kt1 = k_tiles;
        ti.split = 0;
        return ti;
    }
};

// Scale tensor maps view a tile-layout scale buffer as rows of 256 bytes; the 2 KB of one 128-row tile x one
// K-tile (4 x 512 B) is a box of 8 rows starting at row 2 * (tile_row * tile_cols + 4 * kt).
template <class C, class Sched, class Epi>
__global__ void __launch_bounds__(C::THREADS, 1)
    nvf4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                          const __grid_constant__ CUtensorMap tma_sfa, const __grid_constant__ CUtensorMap tma_sfb,
                          const CoreParams cp, Sched sched, const Epi epi) {
    using namespace sm100;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + C::STAGES * C::A_BYTES;
    uint8_t* sSFA = sB + C::STAGES * C::B_BYTES;
    uint8_t* sSFB = sSFA + C::STAGES * C::SFA_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + C::STAGES * C::SFB_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + 1;
    uint64_t* sf_full = tempty + 1;               // per stage: its scales are in TMEM slot `stage`
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sf_full + C::STAGES);
    volatile int* sflag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* esm = sSFB + C::STAGES * C::SFB_BYTES + C::BAR_BYTES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(tfull, 1);
        mbar_init(tempty, 2 * C::EPI_WARPS);
        for (int b = 0; b < C::STAGES; ++b) mbar_init(&sf_full[b], 2);
        *sflag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tma_a);
        prefetch_tmap(&tma_b);
        prefetch_tmap(&tma_sfa);
        prefetch_tmap(&tma_sfb);
    }
    if (warp == 1) { tmem_alloc_pair(tmem_slot, C::TMEM_COLS); tmem_relinquish_pair(); }
    sched_init(sched);
    tc_fence_before();
    cluster_sync();               // barrier inits and the TMEM address visible in both CTAs
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int num_tiles = sched.num_tiles();
    const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = cluster; t < num_tiles && ok; t += clusters) {
                const TileInfo ti = sched.tile(t);
                const int a_row = ti.a_row + (int)rank * C::BM;
                const int sfa_row0 = 2 * ((2 * ti.mb + (int)rank) * cp.tile_cols);
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, sflag, kErrTimeoutProducer)) { ok = false; break; }
                    const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], C::PAIR_TX);
                    tma_load_2d_pair(sA + stage * C::A_BYTES, &tma_a, fb, kt * C::KT_BYTES, a_row);
                    tma_load_2d_pair(sB + stage * C::B_BYTES, &tma_b, fb, kt * C::KT_BYTES,
                                     ti.b_row + (int)rank * (C::BN / 2));
                    tma_load_2d_pair(sSFA + stage * C::SFA_BYTES, &tma_sfa, fb, 0, sfa_row0 + 8 * kt);
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        tma_load_2d_pair(sSFB + stage * C::SFB_BYTES + h * 2048, &tma_sfb, fb, 0,
                                         2 * ((ti.sfb_tile0 + h) * cp.tile_cols) + 8 * kt);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            // Do not leave while the leader's commits for the last stages may still arrive on this CTA's barriers
            // (a slot never filled passes at once: its barrier is still in its first phase).
            for (int i = 0; i < C::STAGES && ok; ++i) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, sflag, kErrTimeoutProducer)) break;
                if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader only) ----------------
        if (rank == 0 && lane == 0) {
            int stage = 0;
            uint32_t phase = 0, aphase = 0;
            bool ok = true;
            const uint32_t sfa_col = tmem + (uint32_t)C::SF_COL0;
            const uint32_t sfb_col = sfa_col + C::SF_COLS_A;
            const uint32_t idesc = idesc_nvf4(C::PAIR_M, C::BN);
            const uint32_t tfull_own = smem_u32(tfull), tfull_peer = mapa_shared(smem_u32(tfull), 1);
            for (int t = cluster; t < num_tiles && ok; t += clusters) {
                const TileInfo ti = sched.tile(t);
                if (!mbar_wait_cluster(tempty, aphase ^ 1u, sflag, kErrTimeoutMma)) break;
                tc_fence_after();
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!mbar_wait(&full[stage], phase, sflag, kErrTimeoutMma)) { ok = false; break; }
                    tc_fence_after();
                    const int nks = min(4, cp.tile_cols - kt * 4);
                    const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
                    const uint32_t acc0 = kt != ti.kt0 ? 1u : 0u;
                    if (!mbar_wait(&sf_full[stage], phase, sflag, kErrTimeoutMma)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t so = (uint32_t)(stage * (C::SF_COLS_A + C::SF_COLS_B));
                    for (int j = 0; j < nks; ++j)
                        mma_nvf4_pair(tmem, desc_kmajor_sw128(a_base + 32 * j), desc_kmajor_sw128(b_base + 32 * j),
                                      idesc, sfa_col + so + 4 * j, sfb_col + so + 8 * j, (acc0 | j) != 0 ? 1u : 0u);
                    const uint32_t eb = smem_u32(&empty[stage]);
                    tc_commit_pair(eb);
                    tc_commit_pair(mapa_shared(eb, 1));
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit_pair(tfull_own);
                tc_commit_pair(tfull_peer);
                aphase ^= 1u;
            }
        }
    } else if (warp < 4) {
        // ---------------- scale copiers (leader warps 2, 3) ----------------
        if (rank == 0 && lane == 0) {
            const int part = warp - 2;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            const uint32_t sfa_col = tmem + (uint32_t)C::SF_COL0;
            const uint32_t sfb_col = sfa_col + C::SF_COLS_A;
            for (int t = cluster; t < num_tiles && ok; t += clusters) {
                const TileInfo ti = sched.tile(t);
                for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
                    if (!mbar_wait(&full[stage], phase, sflag, kErrTimeoutMma)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t so = (uint32_t)(stage * (C::SF_COLS_A + C::SF_COLS_B));
                    issue_scale_copies<C, true>(part, min(4, cp.tile_cols - kt * 4), sfa_col + so, sfb_col + so,
                                                smem_u32(sSFA + stage * C::SFA_BYTES),
                                                smem_u32(sSFB + stage * C::SFB_BYTES));
                    tc_commit_pair(smem_u32(&sf_full[stage]));
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else {
        // ---------------- epilogue (both CTAs) ----------------
        const int ew = warp - 4;
        const int quad = warp & 3;
        const int col_base = (ew >> 2) * C::COLS_PER_WARP;
        const int row = quad * 32 + lane;
        const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
        uint32_t aphase = 0;
        for (int t = cluster; t < num_tiles; t += clusters) {
            TileInfo ti = sched.tile(t);
            ti.a_row += (int)rank * C::BM;
            if (!mbar_wait_cluster(tfull, aphase, sflag, kErrTimeoutEpilogue)) break;
            tc_fence_after();
            const uint32_t addr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)col_base;
            uint32_t r[C::CHUNKS][32];
#pragma unroll
            for (int c = 0; c < C::CHUNKS; ++c) tmem_ld_32x32b_x32(addr + 32 * c, r[c]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader);
            epi.template process<C::CHUNKS>(ti, row, col_base, r, esm);
            aphase ^= 1u;
        }
        epi.finish();
    }

    tc_fence_before();
    cluster_sync();               // every MMA done and every remote arrival made before TMEM is freed
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, C::TMEM_COLS);
    }
    if (threadIdx.x == 0 && *sflag != 0) atomicCAS(cp.err, 0, *sflag);
}

// ---------------------------------------------------------------------------------------------------------------
// Host launch helpers
// ---------------------------------------------------------------------------------------------------------------

int make_kmajor_map(CUtensorMap* map, const void* base, long long rows, long long row_bytes, int box_rows);
// Row-major byte matrix [rows, row_bytes] (row_bytes a multiple of 16) in boxes of box_bytes x box_rows, no swizzle.
int make_rows_map(CUtensorMap* map, const void* base, long long rows, long long row_bytes, int box_bytes,
                  int box_rows);
// Tile-layout scale buffer of `bytes` (a multiple of 512) as rows of 256 bytes, boxes of 8 rows (2 KB), no swizzle.
int make_scale_map(CUtensorMap* map, const void* base, long long bytes);

// Clusters of two that can be resident at once (0 if the query fails).
template <class C, class Sched, class Epi>
int pair_clusters_resident() {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * 148, 1, 1);
    cfg.blockDim = dim3(C::THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, nvf4_gemm_pair_kernel<C, Sched, Epi>, &cfg) != cudaSuccess) return 0;
    return n;
}

template <class C, class Sched, class Epi>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& msfa, const CUtensorMap& msfb,
                const CoreParams& cp, const Sched& s, const Epi& e, int tiles, cudaStream_t stream) {
    static std::atomic<int> clusters[64];     // per device; host threads may race to fill it (same value)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVFP4B_ERR_CUDA;
    int resident = clusters[dev].load(std::memory_order_acquire);
    if (resident == 0) {
        cudaError_t err = cudaFuncSetAttribute(nvf4_gemm_pair_kernel<C, Sched, Epi>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (err != cudaSuccess) return record_cuda_error(err);
        resident = pair_clusters_resident<C, Sched, Epi>();
        if (resident <= 0) return record_cuda_error(cudaErrorLaunchOutOfResources);
        clusters[dev].store(resident, std::memory_order_release);
    }
    const int n = tiles < resident ? tiles : resident;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * n, 1, 1);
    cfg.blockDim = dim3(C::THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, nvf4_gemm_pair_kernel<C, Sched, Epi>, ma, mb, msfa, msfb, cp, s, e);
    if (err != cudaSuccess) return record_cuda_error(err);
    return launch_status();
}

template <class C, class Sched, class Epi>
int launch_core(const CUtensorMap& ma, const CUtensorMap& mb, const CoreParams& cp, const Sched& s, const Epi& e,
                int grid, cudaStream_t stream) {
    static std::atomic<bool> attr_done[64];   // per device; host threads may race to set it (idempotent)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev].load(std::memory_order_acquire)) {
        cudaError_t err = cudaFuncSetAttribute(nvf4_gemm_kernel<C, Sched, Epi>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (err != cudaSuccess) return record_cuda_error(err);
        if (dev >= 0 && dev < 64) attr_done[dev].store(true, std::memory_order_release);
    }
    nvf4_gemm_kernel<C, Sched, Epi><<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(ma, mb, cp, s, e);
    return launch_status();
}

}  // namespace nvfp4b
