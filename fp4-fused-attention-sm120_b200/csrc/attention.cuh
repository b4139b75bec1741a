// attention.cuh -- warp-specialised FP4 fused attention forward for sm_100a,
// one 128-row query tile per work item (head_dim 160 and 256, and the S-only
// debug path for every head_dim; attention_pair.cuh covers head_dim <= 128).
//
// Computes, per (batch, head) slice and 128-row query tile,
//     Out = softmax(Q K^T * scale) V
// with Q, K pre-quantised to E2M1 + UE8M0 (block 32 along head_dim) and V in
// FP16 -- the computation of the reference kernel fused_fp4_attention
// (common.h:68-328), re-designed for Blackwell.  The kernel is persistent: one
// CTA per SM walks (slice, query tile) items, and barrier phases and rings run
// on across items.  Roles:
//
//   warp 0      TMA producer: per item the Q tile (double-buffered across
//               items), then K tiles (codes + scale tiles) and V tiles through
//               KST/VST-stage mbarrier rings.
//   warp 1      S issuer (one thread): S_g = Q K_g^T with tcgen05.mma
//               kind::mxf4 block_scale (scales in TMEM, copied with
//               tcgen05.cp).  S is double-buffered: S_{g+2} is issued when the
//               softmax has finished step g, a whole step before it is needed
//               (possibly the next item's first steps, hence the Q buffers).
//   warp 2      P.V issuer (one thread): O += P_g V_g with tcgen05.mma
//               kind::f16 whose A operand (P) is read from its own TMEM
//               columns; on its own warp so it is issued as soon as P_g is
//               ready.
//   warp 3      idle (completes the control warpgroup for setmaxnreg)
//   warps 4-11  two softmax warpgroups; thread = query row = TMEM lane, and
//               each warpgroup owns half of the S columns (and half of O's).
//               Each warp loads the whole S row and forms the row max itself
//               (its partner computes the same value), so the two halves never
//               wait on each other during a step.  Online max/sum in FP32
//               (log2 domain), P stored as FP16 with tcgen05.st, lazy O
//               rescale (only when the row max grows by more than 2^15); at
//               the end of an item the halves exchange their row sums and
//               write O / l for their half of the columns.
//
// TMEM columns (512 allocated): S0 [0,BN), S1 [BN,2BN), O [2BN, 2BN+D),
// P [.., +BN/2), then two groups of Q scale columns and KST stages of K scale
// columns.
//
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records
// FP4ATTN_ETIMEOUT in the device error word, all roles leave their loops,
// in-flight copies and MMAs are drained (bounded), TMEM is freed, and the CTA
// returns.  Nothing traps.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "ptx_sm100.cuh"

namespace fp4attn {

// Lazy O rescale: O and l keep a reference max until a row's max has grown
// past it by more than 2^kLazyRescaleLog2.  P is then at most 2^15, finite in
// FP16 (max 65504), whose relative precision does not depend on magnitude.
constexpr float kLazyRescaleLog2 = 15.0f;

// Device error word: [0] status code, [1] wait site, [2] block x, [3] block y.
__device__ int g_fp4attn_error[4];

template <int D, int BN>
struct FwdCfg {
    static constexpr int BM = 128;                          // query rows per tile (MMA M)
    static constexpr int DP = (D + 63) / 64 * 64;           // head_dim padded to the MMA K step
    static constexpr int QK_ROW = DP / 2;                   // bytes per packed code row
    static constexpr int CW = QK_ROW == 96 ? 32 : QK_ROW;   // swizzle chunk of a code row
    static constexpr int NCH = QK_ROW / CW;
    static constexpr int KSTEPS = DP / 64;                  // mxf4 MMAs per S tile
    static constexpr int VCW = D == 32 ? 64 : 128;          // swizzle chunk of a V row (bytes)
    static constexpr int VCH = (2 * D + VCW - 1) / VCW;     // V chunks (TMA boxes) per tile
    static constexpr int SFA_ATOMS = (DP + 127) / 128;      // 512-B scale atoms per 128-row tile
    static constexpr int SFB_ATOMS = BN == 128 ? SFA_ATOMS : (DP + 255) / 256;
    static constexpr int SFB_COLS = 4 * SFB_ATOMS;
    static constexpr int KST = D > 128 && BN == 128 ? 2 : 3;  // (TMEM: K scale columns per stage)
    static constexpr int VST = D > 128 && BN == 128 ? 2 : 3;
    // TMEM
    static constexpr int S_COL = 0;
    static constexpr int O_COL = 2 * BN;
    static constexpr int P_COL = O_COL + D;                 // BN/2 columns of FP16 pairs
    static constexpr int SFA_COL = P_COL + BN / 2;
    static constexpr int SFB_COL = SFA_COL + 2 * 4 * SFA_ATOMS;  // Q scales: two buffers (alternate items)
    static constexpr int TMEM_USED = SFB_COL + KST * SFB_COLS;
    static_assert(TMEM_USED <= 512, "TMEM budget exceeded");
    static_assert(D % 32 == 0 && D <= 256, "head_dim");
    static_assert(BN == 128 || BN == 64, "BN");
    // shared memory (offsets from a 1024-aligned base)
    static constexpr int Q_BYTES = BM * QK_ROW;
    static constexpr int QSF_BYTES = SFA_ATOMS * 512;
    static constexpr int K_BYTES = BN * QK_ROW;
    static constexpr int KSF_BYTES = SFB_ATOMS * 512;
    static constexpr int V_BYTES = VCH * BN * VCW;
    static constexpr int align1k(int x) { return (x + 1023) / 1024 * 1024; }
    // Q and its scale tile are double-buffered (alternate work items), so the
    // next item's Q can land while the current item's S MMAs still read theirs.
    static constexpr int Q_STRIDE = align1k(Q_BYTES);
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_QSF = OFF_Q + 2 * Q_STRIDE;
    static constexpr int OFF_K = align1k(OFF_QSF + 2 * QSF_BYTES);
    static constexpr int K_STRIDE = align1k(K_BYTES);
    static constexpr int OFF_KSF = OFF_K + KST * K_STRIDE;
    static constexpr int OFF_V = align1k(OFF_KSF + KST * KSF_BYTES);
    static constexpr int V_STRIDE = align1k(V_BYTES);
    static constexpr int OFF_REDL = OFF_V + VST * V_STRIDE;    // [2 halves][128 rows] f32 row sums
    // Output staging: per softmax warp two buffers of 32 rows x OCH_E columns
    // (sized for FP32), written swizzled and sent out by TMA stores.
    static constexpr int OCH_E = (D / 2) % 32 == 0 ? 32 : 16;
    static constexpr int OST_BYTES = 32 * OCH_E * 4;
    static constexpr int OFF_OST = OFF_REDL + 2 * 128 * 4;
    static constexpr int OFF_BAR = OFF_OST + 8 * 2 * OST_BYTES;
    // q_full[2], q_empty[2], K ring, V ring, s_full[2], p_full[2], pv_done, drain, l_ready[4]
    static constexpr int NUM_BARS = 4 + 2 * KST + 2 * VST + 2 + 2 + 1 + 1 + 4;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 1024;  // +1024 for base alignment
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget exceeded");
};

struct FwdArgs {
    int seq_q, seq_k;
    int nq_tiles, nk_tiles;
    int n_items;               // work items = nq_tiles * slices (one 128-row query tile each)
    int q_sf_tiles;            // 128-row scale tiles per slice in q_sf (>= nq_tiles)
    float scale_log2;          // softmax_scale * log2(e)
    void* out;                 // [slices, seq_q, D] (attention) or [slices, seq_q, seq_k] FP32 (scores)
    const uint8_t* q_sf;       // [slices][q_sf_tiles][QSF_BYTES]
    const uint8_t* k_sf;       // [slices][nk_tiles][KSF_BYTES]
    unsigned long long timeout_ns;
    int causal;                // 1: query i sees keys j <= i + causal_off only (attention, not scores)
    int causal_off;            // seq_k - seq_q (bottom-right alignment)
    int scores_tma;            // scores: 1 if tm_o maps S (seq_k % 4 == 0) and S goes out by TMA stores
    // The two-query-tile kernel's schedule (PairArgs): query tiles per item,
    // key partitions and their partial results.
    int qtiles, n_pairs, kparts, nk_part;
    float2* part_ml;
    float* part_o;
    unsigned* part_count;
    // In-kernel Q quantisation (fp4attn_forward_fused_q): FP16 Q and the scale rule.
    const void* q_in;
    int ocp_mode;
    // fp4attn_forward_lse: per query row the natural-log log-sum-exp of the
    // scaled scores, [slices][seq_q] FP32 (two-query-tile kernel only).
    float* lse;
};

// Work item r of this CTA's static schedule for the one-tile kernel: (slice,
// query tile) and its number of key steps.  Without a mask items go in slice
// order (a slice's K/V stay in L2 while its tiles run); with the causal mask a
// tile needs keys only up to its last row, so items go heaviest first (last
// tiles first) and are dealt to the CTAs in a snake order.
struct TileItem {
    int slice, qt, nk;
    bool valid;
};

template <int BN>
__device__ __forceinline__ TileItem tile_item(const FwdArgs& a, bool causal, int r)
{
    const int G = gridDim.x, b = blockIdx.x;
    TileItem it;
    if (causal) {
        const int w = r * G + ((r & 1) ? G - 1 - b : b);
        const int slices = a.n_items / a.nq_tiles;
        it.valid = w < a.n_items;
        it.slice = w % slices;
        it.qt = a.nq_tiles - 1 - w / slices;
        const int hi = min(it.qt * 128 + 127, a.seq_q - 1) + a.causal_off;  // last key any row sees
        it.nk = hi < 0 ? 1 : min(a.nk_tiles, hi / BN + 1);
    } else {
        const int w = r * G + b;
        it.valid = w < a.n_items;
        it.slice = w / a.nq_tiles;
        it.qt = w % a.nq_tiles;
        it.nk = a.nk_tiles;
    }
    return it;
}

enum WaitSite : int {
    kSiteQFull = 1,
    kSiteKFull,
    kSiteKEmpty,
    kSiteVFull,
    kSiteVEmpty,
    kSiteSFull,
    kSitePFull,
    kSitePvDone,
    kSiteDrain,
    kSiteSFree,
    kSiteQEmpty,
    kSitePartDone,
};

struct WaitCtx {
    volatile int* abort_flag;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ void record_timeout(int site)
{
    if (atomicCAS(&g_fp4attn_error[0], 0, 4 /*FP4ATTN_ETIMEOUT*/) == 0) {
        g_fp4attn_error[1] = site;
        g_fp4attn_error[2] = blockIdx.x;
        g_fp4attn_error[3] = blockIdx.y;
    }
}

// Bounded wait for the phase of `bar` with parity `parity`.  Returns false if
// another role of this CTA already gave up, or if the bound expires (then it
// raises the CTA's abort flag and records the site).
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, const WaitCtx& w, int site)
{
    if (ptx::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = ptx::globaltimer_ns();
    for (uint32_t it = 1; it < (1u << 30); ++it) {
        if (ptx::mbar_try_wait(bar, parity)) return true;
        if ((it & 31u) == 0u) {
            if (*w.abort_flag) return false;
            if (ptx::globaltimer_ns() - t0 > w.timeout_ns) break;
        }
    }
    *w.abort_flag = 1;
    record_timeout(site);
    return false;
}

// Drain wait used on the way out: ignores the abort flag, bounded by `ns`.
__device__ __forceinline__ void drain_phase(uint64_t* bar, uint32_t parity, unsigned long long ns)
{
    const uint64_t t0 = ptx::globaltimer_ns();
    for (uint32_t it = 0; it < (1u << 30); ++it) {
        if (ptx::mbar_try_wait(bar, parity)) return;
        if ((it & 31u) == 0u && ptx::globaltimer_ns() - t0 > ns) {
            record_timeout(kSiteDrain);
            return;
        }
    }
}

// Thread layout: 384 threads = 3 warpgroups.  Each SM sub-partition has its
// own quarter of the register file and hosts one warp of every warpgroup, so
// at launch every thread gets 168 registers (3 x 168 x 32 <= 16384).  The
// control warpgroup then gives registers back (setmaxnreg.dec to kCtlRegs) and
// the two softmax warpgroups take them (setmaxnreg.inc to kSmRegs):
// 128 x 80 + 256 x 208 = 63,488 <= 384 x 168 = 64,512, and per sub-partition
// 80 + 2 x 208 = 496 registers x 32 lanes <= 16,384.  The host checks the
// launch register count before every launch (a shortfall would make
// setmaxnreg.inc wait for registers that never free up).
constexpr int kFwdThreads = 384;
constexpr int kCtlRegs = 80;
constexpr int kSmRegs = 208;
constexpr int kLaunchRegs = 168;
static_assert(128 * kCtlRegs + 256 * kSmRegs <= kFwdThreads * kLaunchRegs, "register split exceeds the launch pool");
static_assert((kCtlRegs + 2 * kSmRegs) * 32 <= 16384, "register split exceeds a sub-partition");

template <int D, int BN, typename OutT, bool kScores, int kPoly8 = 3>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fp4_attention_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                             const FwdArgs args)
{
    using C = FwdCfg<D, BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + C::OFF_Q;
    uint8_t* sQsf = smem + C::OFF_QSF;
    uint8_t* sK = smem + C::OFF_K;
    uint8_t* sKsf = smem + C::OFF_KSF;
    uint8_t* sV = smem + C::OFF_V;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* q_full = bars;              // [2] Q buffer b loaded (TMA)
    uint64_t* q_empty = bars + 2;         // [2] the S MMAs of Q buffer b's item are done (tcgen05.commit)
    uint64_t* k_full = bars + 4;
    uint64_t* k_empty = k_full + C::KST;
    uint64_t* v_full = k_empty + C::KST;
    uint64_t* v_empty = v_full + C::VST;
    uint64_t* s_full = v_empty + C::VST;  // S_j computed (tcgen05.commit)
    uint64_t* p_full = s_full + 2;        // step j done: S_j read, P_j stored, O rescaled (256 threads)
    uint64_t* pv_done = p_full + 2;       // O += P_j V_j complete (tcgen05.commit)
    uint64_t* drain_bar = pv_done + 1;
    uint64_t* l_ready = drain_bar + 1;    // [lane quarter] both halves' row sums are in red_l (64 threads)

    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // Persistent: this CTA runs items tile_item(args, causal, r) for r = 0, 1,
    // ...; barrier phases and ring indices run on across items (global step g).
    const bool causal = !kScores && args.causal;
    const int rounds = (args.n_items + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; b++) {
            ptx::mbar_init(&q_full[b], 1);
            ptx::mbar_init(&q_empty[b], 1);
        }
        for (int i = 0; i < C::KST; i++) {
            ptx::mbar_init(&k_full[i], 1);
            ptx::mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < C::VST; i++) {
            ptx::mbar_init(&v_full[i], 1);
            ptx::mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            ptx::mbar_init(&s_full[i], 1);
            ptx::mbar_init(&p_full[i], 256);
        }
        ptx::mbar_init(pv_done, 1);
        ptx::mbar_init(drain_bar, 2);  // one commit from each MMA issuer
        for (int q = 0; q < 4; q++) ptx::mbar_init(&l_ready[q], 64);
        abort_sh = 0;
        ptx::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        ptx::prefetch_tmap(&tm_q);
        ptx::prefetch_tmap(&tm_k);
        if (!kScores) {
            ptx::prefetch_tmap(&tm_v);
            ptx::prefetch_tmap(&tm_o);
        }
    }
    if (warp == 1) {
        ptx::tmem_alloc(&tmem_base_sh, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    const WaitCtx wctx{&abort_sh, args.timeout_ns};
    // Everything above overlaps the quantiser's tail when this grid was
    // launched as its programmatic dependent; from here on the workspace it
    // wrote is read.
    ptx::grid_dependency_wait();

    if (warp < 4) {
        ptx::setmaxnreg_dec<kCtlRegs>();
        if (warp == 0) {
            // -------------------------------------------------------- producer
            if (lane == 0) {
                int it = 0, kv = 0, k_issued = 0, v_issued = 0;
                bool ok = true;
                for (int r = 0; ok && r < rounds; r++) {
                    const TileItem item = tile_item<BN>(args, causal, r);
                    if (!item.valid) continue;
                    const int qb = it & 1;
                    // Q buffer qb last held item it-2; its S MMAs must be done.
                    if (it >= 2 && !wait_phase(&q_empty[qb], ((it >> 1) - 1) & 1, wctx, kSiteQEmpty)) break;
                    ptx::mbar_arrive_expect_tx(&q_full[qb], C::Q_BYTES + C::QSF_BYTES);
#pragma unroll
                    for (int c = 0; c < C::NCH; c++)
                        ptx::tma_load_3d(sQ + qb * C::Q_STRIDE + c * C::BM * C::CW, &tm_q, &q_full[qb], c * C::CW,
                                         item.qt * C::BM, item.slice);
                    ptx::bulk_load(sQsf + qb * C::QSF_BYTES,
                                   args.q_sf + (static_cast<size_t>(item.slice) * args.q_sf_tiles + item.qt) * C::QSF_BYTES,
                                   C::QSF_BYTES, &q_full[qb]);
                    it++;
                    for (int j = 0; j < item.nk; j++, kv++) {
                        const int ks = kv % C::KST;
                        if (kv >= C::KST && !wait_phase(&k_empty[ks], ((kv / C::KST) - 1) & 1, wctx, kSiteKEmpty)) {
                            ok = false;
                            break;
                        }
                        ptx::mbar_arrive_expect_tx(&k_full[ks], C::K_BYTES + C::KSF_BYTES);
#pragma unroll
                        for (int c = 0; c < C::NCH; c++)
                            ptx::tma_load_3d(sK + ks * C::K_STRIDE + c * BN * C::CW, &tm_k, &k_full[ks], c * C::CW,
                                             j * BN, item.slice);
                        ptx::bulk_load(sKsf + ks * C::KSF_BYTES,
                                       args.k_sf + (static_cast<size_t>(item.slice) * args.nk_tiles + j) * C::KSF_BYTES,
                                       C::KSF_BYTES, &k_full[ks]);
                        k_issued = kv + 1;
                        if (!kScores) {
                            const int vs = kv % C::VST;
                            if (kv >= C::VST && !wait_phase(&v_empty[vs], ((kv / C::VST) - 1) & 1, wctx, kSiteVEmpty)) {
                                ok = false;
                                break;
                            }
                            ptx::mbar_arrive_expect_tx(&v_full[vs], C::V_BYTES);
#pragma unroll
                            for (int c = 0; c < C::VCH; c++)
                                ptx::tma_load_3d(sV + vs * C::V_STRIDE + c * BN * C::VCW, &tm_v, &v_full[vs],
                                                 c * (C::VCW / 2), j * BN, item.slice);
                            v_issued = kv + 1;
                        }
                    }
                }
                // Every load this thread issued must land before the CTA exits
                // (each ring's loads are at most its depth ahead of their use).
                const unsigned long long drain_ns = 2ull * args.timeout_ns;
                for (int i = it - 2 < 0 ? 0 : it - 2; i < it; i++) drain_phase(&q_full[i & 1], (i >> 1) & 1, drain_ns);
                for (int i = k_issued - C::KST < 0 ? 0 : k_issued - C::KST; i < k_issued; i++)
                    drain_phase(&k_full[i % C::KST], (i / C::KST) & 1, drain_ns);
                for (int i = v_issued - C::VST < 0 ? 0 : v_issued - C::VST; i < v_issued; i++)
                    drain_phase(&v_full[i % C::VST], (i / C::VST) & 1, drain_ns);
            }
            __syncwarp();
        } else if (warp == 1) {
            // -------------------------------------------------------- S = Q K^T issuer
            if (lane == 0) {
                constexpr uint32_t qk_layout = ptx::swizzle_mode_for_bytes(C::CW);
                // Descriptors are built once; per MMA only the 16-byte-unit start
                // address in the low bits moves.
                const uint64_t qdesc0 = ptx::make_sdesc(ptx::smem_u32(sQ), 16, 8 * C::CW, qk_layout);
                const uint64_t kdesc0 = ptx::make_sdesc(ptx::smem_u32(sK), 16, 8 * C::CW, qk_layout);
                const uint64_t sfdesc0 = ptx::make_sdesc(ptx::smem_u32(sKsf), 0, 128, ptx::kSwizzleNone);
                const uint64_t qsfdesc0 = ptx::make_sdesc(ptx::smem_u32(sQsf), 0, 128, ptx::kSwizzleNone);
                // Global step g (S buffer g & 1, K ring index g); item counter it (Q buffer it & 1).
                int g = 0, it = 0;
                bool ok = true;
                for (int r = 0; ok && r < rounds; r++) {
                    const TileItem item = tile_item<BN>(args, causal, r);
                    if (!item.valid) continue;
                    const int qb = it & 1;
                    const uint32_t sfa = tmem + C::SFA_COL + qb * 4 * C::SFA_ATOMS;
                    for (int j = 0; j < item.nk; j++, g++) {
                        // S_g reuses S_{g-2}'s buffer once the softmax is done with
                        // step g-2; it is needed only a whole step later.
                        if (g >= 2) {
                            if (!wait_phase(&p_full[g & 1], ((g >> 1) - 1) & 1, wctx, kSitePFull)) {
                                ok = false;
                                break;
                            }
                            ptx::tc_fence_after();
                        }
                        if (j == 0) {
                            // This item's Q and its scales (the item that last used
                            // buffer qb finished its S MMAs before Q was loaded).
                            if (!wait_phase(&q_full[qb], (it >> 1) & 1, wctx, kSiteQFull)) {
                                ok = false;
                                break;
                            }
                            ptx::tc_fence_after();
#pragma unroll
                            for (int at = 0; at < C::SFA_ATOMS; at++)
                                ptx::tc_cp_32x128b_warpx4(
                                    sfa + 4 * at, qsfdesc0 + static_cast<uint64_t>((qb * C::QSF_BYTES + 512 * at) >> 4));
                        }
                        const int ks = g % C::KST;
                        if (!wait_phase(&k_full[ks], (g / C::KST) & 1, wctx, kSiteKFull)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
                        const uint32_t sfb_base = tmem + C::SFB_COL + ks * C::SFB_COLS;
#pragma unroll
                        for (int at = 0; at < C::SFB_ATOMS; at++)
                            ptx::tc_cp_32x128b_warpx4(sfb_base + 4 * at,
                                                      sfdesc0 + static_cast<uint64_t>((ks * C::KSF_BYTES + 512 * at) >> 4));
                        const uint32_t s_tmem = tmem + C::S_COL + (g & 1) * BN;
                        const uint64_t kdesc = kdesc0 + static_cast<uint64_t>((ks * C::K_STRIDE) >> 4);
                        const uint64_t qdesc = qdesc0 + static_cast<uint64_t>((qb * C::Q_STRIDE) >> 4);
#pragma unroll
                        for (int kk = 0; kk < C::KSTEPS; kk++) {
                            const int off = kk * 32, ch = off / C::CW, in = off % C::CW;
                            const uint32_t sf_id = 2u * (kk & 1);
                            ptx::mma_mxf4(s_tmem, qdesc + static_cast<uint64_t>((ch * C::BM * C::CW + in) >> 4),
                                          kdesc + static_cast<uint64_t>((ch * BN * C::CW + in) >> 4),
                                          ptx::idesc_mxf4(128, BN, sf_id, sf_id), (sfa + 4 * (kk >> 1)) | (sf_id << 30),
                                          (sfb_base + (BN == 128 ? 4 : 2) * (kk >> 1)) | (sf_id << 30), kk > 0 ? 1u : 0u);
                        }
                        ptx::tc_commit(&s_full[g & 1]);
                        ptx::tc_commit(&k_empty[ks]);
                    }
                    if (!ok) break;
                    ptx::tc_commit(&q_empty[qb]);  // the producer may load Q buffer qb again
                    it++;
                }
                // Drain every tcgen05 op this thread issued before TMEM is freed.
                ptx::tc_commit(drain_bar);
                drain_phase(drain_bar, 0, 2ull * args.timeout_ns);
            }
            __syncwarp();
        } else if (warp == 2) {
            // -------------------------------------------------------- O += P V issuer
            // On its own warp (and SM sub-partition), so P.V is issued the moment
            // P_j is ready instead of queueing behind the S issue.
            if (lane == 0) {
                if (!kScores) {
                    constexpr uint32_t v_layout = ptx::swizzle_mode_for_bytes(C::VCW);
                    const uint64_t vdesc0 = ptx::make_sdesc(ptx::smem_u32(sV), BN * C::VCW, 8 * C::VCW, v_layout);
                    constexpr uint32_t idesc_pv = ptx::idesc_f16(128, D, true);
                    int g = 0;  // global step: p_full phase and V ring index
                    bool ok = true;
                    for (int r = 0; ok && r < rounds; r++) {
                        const TileItem item = tile_item<BN>(args, causal, r);
                        if (!item.valid) continue;
                        for (int j = 0; j < item.nk; j++, g++) {
                            if (!wait_phase(&p_full[g & 1], (g >> 1) & 1, wctx, kSitePFull)) {
                                ok = false;
                                break;
                            }
                            const int vs = g % C::VST;
                            if (!wait_phase(&v_full[vs], (g / C::VST) & 1, wctx, kSiteVFull)) {
                                ok = false;
                                break;
                            }
                            ptx::tc_fence_after();
                            const uint64_t vdesc = vdesc0 + static_cast<uint64_t>((vs * C::V_STRIDE) >> 4);
                            // The first step of an item starts O afresh.
#pragma unroll
                            for (int kk = 0; kk < BN / 16; kk++)
                                ptx::mma_f16_ts(tmem + C::O_COL, tmem + C::P_COL + kk * 8,
                                                vdesc + static_cast<uint64_t>((kk * 16 * C::VCW) >> 4), idesc_pv,
                                                (j > 0 || kk > 0) ? 1u : 0u);
                            ptx::tc_commit(&v_empty[vs]);
                            ptx::tc_commit(pv_done);
                        }
                    }
                }
                ptx::tc_commit(drain_bar);
                drain_phase(drain_bar, 0, 2ull * args.timeout_ns);
            }
            __syncwarp();
        }
    } else {
        ptx::setmaxnreg_inc<kSmRegs>();
        // ------------------------------------------------------------ softmax warpgroups
        constexpr int HC = BN / 2;                 // S columns per warpgroup
        constexpr int NT = HC / 32;                // 32-column chunks per warpgroup
        constexpr int HD = D / 2;                  // O columns per warpgroup
        constexpr int OCH = HD % 32 == 0 ? 32 : 16;  // O column chunk
        const int half = (warp - 4) / 4;           // which half of the columns
        const int wq = warp & 3;                   // TMEM lane quarter this warp may access
        const int row = wq * 32 + lane;            // query row within the tile
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        float* red_l = reinterpret_cast<float*>(smem + C::OFF_REDL);
        const float c = args.scale_log2;
        bool ok = true;
        auto load_s = [&](int g, uint32_t (&buf)[NT][32]) {
            const uint32_t s_tm = tmem + lane_off + C::S_COL + (g & 1) * BN + half * HC;
#pragma unroll
            for (int t = 0; t < NT; t++) ptx::tmem_ld32(s_tm + 32 * t, buf[t]);
        };
        int g0 = 0;  // global step of the current item's first step (S buffer and barrier phases)
        int items_done = 0;  // phase of l_ready
        int sbox = 0;        // scores: boxes this warp has stored (staging buffer alternation)
        uint8_t* ost = smem + C::OFF_OST + (warp - 4) * 2 * C::OST_BYTES;
        for (int r = 0; ok && r < rounds; r++) {
        const TileItem item = tile_item<BN>(args, causal, r);
        if (!item.valid) continue;
        const int slice = item.slice, q0 = item.qt * C::BM, nk = item.nk;
        float m = -INFINITY, l = 0.f;
        if (kScores) {
            for (int j = 0; j < nk; j++) {
                const int g = g0 + j;
                if (!__all_sync(0xffffffffu, wait_phase(&s_full[g & 1], (g >> 1) & 1, wctx, kSiteSFull))) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                uint32_t sr[NT][32];
                load_s(g, sr);
                ptx::tc_wait_ld();
                if (args.scores_tma) {
                    // This warp's 32 rows x HC columns of S in OCH_E-column boxes:
                    // each staged swizzled like the TMA box and stored by lane 0;
                    // rows past seq_q and columns past seq_k are clipped by the map.
                    constexpr int OE = C::OCH_E, OB = OE * 4;
#pragma unroll
                    for (int b = 0; b < HC / OE; b++, sbox++) {
                        uint8_t* buf = ost + (sbox & 1) * C::OST_BYTES;
                        if (sbox >= 2) {
                            // The store that last read this buffer must be done with it.
                            if (lane == 0) ptx::bulk_wait_group_read<1>();
                            __syncwarp();
                        }
#pragma unroll
                        for (int u = 0; u < OB / 16; u++) {
                            const int c = b * OE + 4 * u;  // first column of this 16-byte unit
                            const int pu = OB == 128 ? (u ^ (lane & 7)) : (u ^ ((lane >> 1) & 3));
                            *reinterpret_cast<uint4*>(buf + lane * OB + pu * 16) =
                                make_uint4(sr[c / 32][c % 32], sr[c / 32][c % 32 + 1], sr[c / 32][c % 32 + 2],
                                           sr[c / 32][c % 32 + 3]);
                        }
                        ptx::fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            ptx::tma_store_3d(&tm_o, buf, j * BN + half * HC + b * OE, q0 + wq * 32, slice);
                            ptx::bulk_commit_group();
                        }
                    }
                } else {
                const int valid = args.seq_k - j * BN - half * HC;
                const int grow = q0 + row;
                if (grow < args.seq_q) {
                    float* dst = reinterpret_cast<float*>(args.out) +
                                 (static_cast<size_t>(slice) * args.seq_q + grow) * args.seq_k +
                                 static_cast<size_t>(j) * BN + half * HC;
#pragma unroll
                    for (int t = 0; t < NT; t++)
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (32 * t + i < valid) dst[32 * t + i] = __uint_as_float(sr[t][i]);
                }
                }
                ptx::tc_fence_before();
                ptx::mbar_arrive(&p_full[g & 1]);  // done with S_g: its buffer may be reused
            }
        } else {
            // Each warp loads the whole S_j row (all BN columns) to form the
            // row max itself -- the partner warp computes the same max from the
            // same values, so the halves never wait on each other -- and then
            // exponentiates only its own half of the columns.
            constexpr int NF = BN / 32;            // 32-column chunks of a full S row
            // Keys this row sees: [0, row_lim) (the causal mask, or all keys).
            const int row_lim = causal ? min(q0 + row + args.causal_off + 1, args.seq_k) : args.seq_k;
            for (int j = 0; j < nk; j++) {
                const int g = g0 + j;
                if (!__all_sync(0xffffffffu, wait_phase(&s_full[g & 1], (g >> 1) & 1, wctx, kSiteSFull))) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                uint32_t sr[NF][32];
                {
                    const uint32_t s_tm = tmem + lane_off + C::S_COL + (g & 1) * BN;
#pragma unroll
                    for (int t = 0; t < NF; t++) ptx::tmem_ld32(s_tm + 32 * t, sr[t]);
                }
                ptx::tc_wait_ld();
                const int valid = row_lim - j * BN;  // keys of this step this row sees
                if (valid < BN) {
#pragma unroll
                    for (int t = 0; t < NF; t++)
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (32 * t + i >= valid) sr[t][i] = __float_as_uint(-INFINITY);
                }
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int t = 0; t < NF; t++)
#pragma unroll
                    for (int i = 0; i < 32; i += 2)
                        mx4[(i >> 1) & 3] =
                            ptx::fmax3(mx4[(i >> 1) & 3], __uint_as_float(sr[t][i]), __uint_as_float(sr[t][i + 1]));
                const float mx = ptx::fmax3(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3]));
                const float m_new = fmaxf(m, mx * c);
                float alpha = 1.f;
                bool rescale = false;
                if (j == 0) {
                    m = m_new;
                } else if (m_new > m + kLazyRescaleLog2) {
                    alpha = ptx::ex2_approx(m - m_new);
                    m = m_new;
                    rescale = true;
                }
                float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                // A row that has seen no key yet keeps m = -inf; its P is 0.
                const float m_ref = m == -INFINITY ? 0.f : m;
                const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_ref, -m_ref);
                uint32_t pk[NT][16];
                // Exponentials of one 32-column chunk (indices stay compile-time
                // so the row stays in registers).
                auto exps_chunk = [&](const uint32_t (&src)[32], uint32_t (&dst)[16]) {
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float2 x = ptx::ffma2(make_float2(__uint_as_float(src[i]), __uint_as_float(src[i + 1])), c2, nm2);
                        // kPoly8 of every 8 column pairs take 2^x on the FMA pipe,
                        // the rest on MUFU, so both pipes share the exponentials.
                        const float2 p = ((i >> 1) & 7) < kPoly8
                                             ? ptx::exp2_poly3(x)
                                             : make_float2(ptx::ex2_approx(x.x), ptx::ex2_approx(x.y));
                        sum2[(i >> 1) & 1] = ptx::fadd2(sum2[(i >> 1) & 1], p);
                        dst[i / 2] = ptx::pack_half2(p.x, p.y);
                    }
                };
                if (half == 0) {
#pragma unroll
                    for (int t = 0; t < NT; t++) exps_chunk(sr[t], pk[t]);
                } else {
#pragma unroll
                    for (int t = 0; t < NT; t++) exps_chunk(sr[NT + t], pk[t]);
                }
                l = l * alpha + ((sum2[0].x + sum2[1].x) + (sum2[0].y + sum2[1].y));
                if (j > 0) {
                    // PV_{j-1} must be done: it reads the P columns this step
                    // overwrites, and O is rescaled below (waiting every phase
                    // also keeps this barrier's parity unambiguous).
                    if (!__all_sync(0xffffffffu, wait_phase(pv_done, (g - 1) & 1, wctx, kSitePvDone))) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                }
                const uint32_t p_tm = tmem + lane_off + C::P_COL + half * (HC / 2);
#pragma unroll
                for (int t = 0; t < NT; t++) ptx::tmem_st16(p_tm + 16 * t, pk[t]);
                if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
                    for (int t = 0; t < HD / OCH; t++) {
                        const uint32_t o_tm = tmem + lane_off + C::O_COL + half * HD + OCH * t;
                        if constexpr (OCH == 32) {
                            uint32_t o[32];
                            ptx::tmem_ld32(o_tm, o);
                            ptx::tc_wait_ld();
#pragma unroll
                            for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                            ptx::tmem_st32(o_tm, o);
                        } else {
                            uint32_t o[16];
                            ptx::tmem_ld16(o_tm, o);
                            ptx::tc_wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                            ptx::tmem_st16(o_tm, o);
                        }
                    }
                }
                ptx::tc_wait_st();
                ptx::tc_fence_before();
                ptx::mbar_arrive(&p_full[g & 1]);
            }
        }
        if (!kScores && ok) {
            // Exchange the half-row sums through shared memory; the wait is
            // bounded, so a partner that left early cannot hold this warp.
            red_l[half * 128 + row] = l;
            ptx::mbar_arrive(&l_ready[wq]);
            if (!__all_sync(0xffffffffu, wait_phase(&l_ready[wq], items_done & 1, wctx, kSiteSFull))) {
                ok = false;
                break;
            }
            items_done++;
            const float l_tot = l + red_l[(1 - half) * 128 + row];
            // Waits are decided per warp (__all_sync) so that warp-wide steps stay uniform.
            if (__all_sync(0xffffffffu, wait_phase(pv_done, (g0 + nk - 1) & 1, wctx, kSitePvDone))) {
                ptx::tc_fence_after();
                const float inv_l = l_tot > 0.f ? 1.0f / l_tot : 0.f;  // a row that saw no key outputs 0
                // O / l in OCH_E-column chunks: each warp writes its 32 rows
                // to a staging buffer (swizzled like the TMA box, so a warp's
                // 16-byte writes hit distinct banks) and lane 0 stores the box
                // with TMA; rows past seq_q are clipped by the tensor map.
                constexpr int OE = C::OCH_E;
                constexpr int OB = OE * static_cast<int>(sizeof(OutT));  // bytes per staged row (32, 64, 128)
                // The previous item's stores must be done reading the staging buffers.
                if (lane == 0) ptx::bulk_wait_group_read<0>();
                __syncwarp();
#pragma unroll 1
                for (int t = 0; t < HD / OE; t++) {
                    uint32_t o[OE];
                    if constexpr (OE == 32) {
                        ptx::tmem_ld32(tmem + lane_off + C::O_COL + half * HD + OE * t, o);
                    } else {
                        ptx::tmem_ld16(tmem + lane_off + C::O_COL + half * HD + OE * t, o);
                    }
                    ptx::tc_wait_ld();
                    uint8_t* buf = ost + (t & 1) * C::OST_BYTES;
                    if (t >= 2) {
                        // The store that last read this buffer must be done with it.
                        if (lane == 0) ptx::bulk_wait_group_read<1>();
                        __syncwarp();
                    }
                    uint32_t ov[OB / 4];
                    if constexpr (sizeof(OutT) == 4) {
#pragma unroll
                        for (int i = 0; i < OE; i++) ov[i] = __float_as_uint(__uint_as_float(o[i]) * inv_l);
                    } else {
#pragma unroll
                        for (int i = 0; i < OE / 2; i++)
                            ov[i] = ptx::pack_half2(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
                    }
                    // 16-byte unit u of row `lane` sits at unit u ^ (address bits 7 and up):
                    // SWIZZLE_128B / 64B / 32B for 128- / 64- / 32-byte rows.
#pragma unroll
                    for (int u = 0; u < OB / 16; u++) {
                        const int pu = OB == 128 ? (u ^ (lane & 7)) : OB == 64 ? (u ^ ((lane >> 1) & 3)) : (u ^ ((lane >> 2) & 1));
                        *reinterpret_cast<uint4*>(buf + lane * OB + pu * 16) =
                            make_uint4(ov[4 * u], ov[4 * u + 1], ov[4 * u + 2], ov[4 * u + 3]);
                    }
                    ptx::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        ptx::tma_store_3d(&tm_o, buf, half * HD + OE * t, q0 + wq * 32, slice);
                        ptx::bulk_commit_group();
                    }
                }
            } else {
                ok = false;
            }
        }
        g0 += nk;
        }
        // Shared memory must outlive the stores that read it.
        if (lane == 0) ptx::bulk_wait_group<0>();
        __syncwarp();
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

// Evaluates the FMA-pipe exponential used by the softmax on n inputs (pairs),
// so tests can hold it to its error bound.
__global__ void exp2_poly_selftest_kernel(const float2* __restrict__ x, float2* __restrict__ y, int64_t n2)
{
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n2;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = ptx::exp2_poly3(x[i]);
}

// A CTA that waits on an mbarrier nothing completes, so that its bounded wait
// expires: exercises the timeout path (error word + clean exit) on purpose.
__global__ void timeout_selftest_kernel(unsigned long long timeout_ns)
{
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_sh;
    if (threadIdx.x == 0) {
        ptx::mbar_init(&bar, 1);
        abort_sh = 0;
        ptx::fence_mbar_init();
    }
    __syncthreads();
    const WaitCtx w{&abort_sh, timeout_ns};
    if (threadIdx.x == 0) (void)wait_phase(&bar, 0, w, kSiteQFull);
    __syncthreads();
}

}  // namespace fp4attn
