// attention_bwd.cuh -- backward pass of the FP4 fused attention on sm_100a
// (head_dim 32, 64, 96 and 128).
//
// The forward (attention_pair.cuh, attention.cuh) computes, per slice,
//     z = scale * Qq Kq^T,   P = softmax(z) (row-wise),   O = P V
// where Qq, Kq are Q and K after the reference's E2M1 + UE8M0 quantisation
// (common.h:21-48, :108-169) and dequantisation.  The reference is forward
// only; this pass differentiates that computation with the quantiser as a
// straight-through estimator (d Qq / d Q = identity), the usual treatment of
// a rounding step in low-precision training:
//     dV = P^T dO,   dP = dO V^T,   Dd_i = sum_c dO_ic O_ic,
//     dZ = P o (dP - Dd),   dQ = scale * dZ Kq,   dK = scale * dZ^T Qq.
// P is rebuilt from S = Qq Kq^T (the same block-scaled E2M1 MMA as the
// forward) and the forward's per-row log-sum-exp: P = 2^(S c - lse2), with
// c = scale * log2(e) and lse2 = lse * log2(e).
//
// One work item is one 128-key tile of one slice; the kernel is persistent
// (one CTA per SM walks the items).  An item holds its keys' K codes and
// scales, V (FP16) and Kq (BF16) in shared memory and walks the 64-row query
// tiles that see its keys.  Per step, with the keys as the MMA M dimension:
//     S^T  = K Q^T          tcgen05.mma kind::mxf4 block_scale  (M128 N64)
//     dP^T = V dO^T         kind::f16, F16 operands             (M128 N64)
//     dV  += P^T dO         kind::f16, F16, P read from TMEM     (M128 N=D)
//     dK  += dZ^T Qq        kind::f16, BF16                      (M128 N=D)
//     dQ^T = Kq^T dZ^T      kind::f16, BF16, A and B MN-major    (M128 N64)
// dZ carries the softmax scale.  dV and dK accumulate in TMEM over the item's
// steps; each step's dQ^T tile (head_dim rows x 64 queries) is added into the
// FP32 dQ output (cleared by the host first) with coalesced reductions (the
// other key tiles of the slice add theirs).
//
// The tensor core reads both operands of an MMA from shared memory unless A
// is in TMEM; at N = 64 those reads, not the multiply, set the MMA's pace, so
// P goes to TMEM (dV's A) and dQ^T leaves through registers, keeping shared
// memory for the operands that must live there.
//
// Roles (512 threads):
//   warp 0       TMA producer: per item K codes + scale tile, V, Kq; per step
//                (QST-stage ring) Q codes + scale tile, dO, Qq, lse2, Dd.
//   warp 1       S issuer (one thread): S^T and dP^T of step g+1, issued as
//                soon as the gradient warpgroups hold step g's in registers,
//                so the tensor core computes them while the warpgroups work
//                on step g.
//   warp 2       gradient issuer (one thread): dV, dK and dQ^T of step g once
//                its P and dZ are stored.
//                A tcgen05.mma waits at issue until the tensor pipe takes it,
//                and the pipe holds about one instruction beyond the one it
//                runs, so each next MMA must be issued within a few cycles of
//                the last one leaving.  One issuing thread, sharing its
//                sub-partition's issue slots with two gradient warps and the
//                dQ warp, misses that window often enough to leave the pipe
//                idle a third of the time; two issuers keep two instructions
//                waiting.  The two streams touch disjoint TMEM columns and
//                their order is set by the barriers below.
//   warp 3       idle.
//   warps 4-11   two gradient warpgroups; thread = key row = TMEM lane, and
//                warpgroup h owns queries [32h, 32h + 32) of the step.  Each
//                reads its S^T and dP^T columns, forms P and dZ, stores P into
//                TMEM (tcgen05.st) and dZ into shared memory as a 128-byte
//                swizzled row (K-major for dK, MN-major for dQ^T).
//   warps 12-15  dQ warpgroup: thread = head-dim row of dQ^T = TMEM lane.  Per
//                step it reads its dQ^T row and adds it into dQ
//                (red.global.add; a warp covers 32 consecutive head-dim
//                entries of one query row: 128 contiguous bytes).  At the end
//                of an item it writes dV and dK (thread = key row).
//
// TMEM columns (512 allocated): S^T [0,64), dP^T [64,128), dV [128, 128+D),
// dK [128+D, 128+2D), dQ^T [128+2D, +64), P [.., +32) (FP16 pairs), K scales
// (4), Q scales (4).
//
// Every mbarrier wait is bounded (globaltimer) as in the forward kernels: on
// expiry the CTA records FP4ATTN_ETIMEOUT, every role leaves its loop,
// in-flight copies and MMAs are drained (bounded), TMEM is freed and the CTA
// returns.  Roles synchronise through mbarriers only, so a role that gives up
// cannot strand another one.
#pragma once

#include <cuda_bf16.h>

#include <climits>
#include <type_traits>

#include "attention.cuh"
#include "quantize.cuh"

namespace fp4attn {

template <int D>
struct BwdCfg {
    static_assert(D == 32 || D == 64 || D == 96 || D == 128, "the backward kernel covers head_dim 32 to 128");
    static constexpr int THREADS = 512;
    static constexpr int BK = 128;                  // keys per item (MMA M)
    static constexpr int BQ = 64;                   // queries per step
    static constexpr int DP = (D + 63) / 64 * 64;   // head_dim padded to the mxf4 K step (zero codes beyond D)
    static constexpr int QK_ROW = DP / 2;           // bytes per packed code row (swizzle = row)
    static constexpr int KSTEPS = DP / 64;          // mxf4 MMAs per S^T tile (K = 64 each)
    // 16-bit operands (V, dO, Qq, Kq) in chunks of CHE columns, CB-byte
    // swizzled rows: 64 columns (128-byte swizzle) where 64 divides head_dim,
    // else 32 (64-byte swizzle).
    static constexpr int CHE = D % 64 == 0 ? 64 : 32;
    static constexpr int CB = 2 * CHE;
    static constexpr uint32_t CSW = CB == 128 ? ptx::kSwizzle128B : ptx::kSwizzle64B;
    static constexpr int DCH = D / CHE;             // chunks of a 16-bit row
    static constexpr int KPC = CHE / 16;            // K = 16 MMA steps per chunk
    static constexpr int QST = 3;                   // query stages
    // TMEM
    static constexpr int S_COL = 0;
    static constexpr int DP_COL = 64;
    static constexpr int DV_COL = 128;
    static constexpr int DK_COL = DV_COL + D;
    static constexpr int DQ_COL = DK_COL + D;
    static constexpr int P_COL = DQ_COL + 64;
    static constexpr int SFA_COL = P_COL + 32;
    // One Q scale group: step g+1's scales are copied in after S of step g
    // has completed (its gradient warpgroups have read it).
    static constexpr int SFB_COL = SFA_COL + 4;
    static constexpr int TMEM_USED = SFB_COL + 4;
    static_assert(TMEM_USED <= 512, "TMEM budget exceeded");
    // shared memory (offsets from a 1024-aligned base)
    static constexpr int align1k(int x) { return (x + 1023) / 1024 * 1024; }
    static constexpr int K_BYTES = BK * QK_ROW;
    static constexpr int SF_BYTES = 512;
    static constexpr int OFF_K = 0;
    static constexpr int OFF_KSF = align1k(K_BYTES);
    static constexpr int OFF_V = align1k(OFF_KSF + SF_BYTES);
    static constexpr int V_BYTES = DCH * BK * CB;
    static constexpr int OFF_KQ = OFF_V + V_BYTES;
    // Kq: 128 / CHE chunks, the M = 128 of the dQ^T MMA; chunks past head_dim
    // are zero and so are those dQ^T rows.
    static constexpr int KQ_CHUNKS = 128 / CHE;
    static constexpr int KQ_BYTES = KQ_CHUNKS * BK * CB;
    static constexpr int OFF_STAGE = OFF_KQ + KQ_BYTES;
    // one query stage
    static constexpr int SQ_Q = 0;
    static constexpr int Q_BYTES = BQ * QK_ROW;
    static constexpr int SQ_QSF = align1k(Q_BYTES);
    static constexpr int SQ_DO = align1k(SQ_QSF + SF_BYTES);
    static constexpr int DO_BYTES = DCH * BQ * CB;
    static constexpr int SQ_QQ = SQ_DO + DO_BYTES;
    static constexpr int SQ_LSE = SQ_QQ + DO_BYTES;
    static constexpr int SQ_DD = SQ_LSE + BQ * 4;
    static constexpr int STAGE_BYTES = align1k(SQ_DD + BQ * 4);
    static constexpr int STAGE_TX = Q_BYTES + SF_BYTES + 2 * DO_BYTES + 2 * BQ * 4;
    static constexpr int KV_TX = K_BYTES + SF_BYTES + 2 * V_BYTES;  // K codes, scales, V, Kq (D columns)
    // dZ: 128 key rows x 64 queries (BF16), 128-byte swizzled rows
    static constexpr int OFF_DS = OFF_STAGE + QST * STAGE_BYTES;
    static constexpr int OFF_BAR = OFF_DS + BK * 128;
    // kv_full, kv_empty, q_full[QST], q_empty[QST], s_full, s_free, ds_full,
    // ds_free, dq_full, dq_free, acc_full, acc_free, drain (S issuer), drain
    // (gradient issuer)
    static constexpr int NUM_BARS = 2 + 2 * QST + 10;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 1024;
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget exceeded");
};

struct BwdArgs {
    int seq_q, seq_k;
    int sq_pad;                // seq_q rounded up to BQ (row pitch of lse2, dd and the dQ accumulator)
    int nq_tiles, nk_tiles;    // 64-row query tiles, 128-row key tiles per slice
    int n_items;               // slices * nk_tiles
    int slices;
    float scale_log2;          // softmax_scale * log2(e)
    float scale;               // softmax_scale
    const uint8_t* q_sf;       // [slices][nq_tiles][512]  (64-row scale tiles)
    const uint8_t* k_sf;       // [slices][nk_tiles][512]  (128-row scale tiles)
    const float* nlse2;        // [slices][sq_pad]: -lse * log2(e); -inf on padding rows
    const float* ndd;          // [slices][sq_pad]: -rowsum(dO o O); 0 on padding rows
    float* dq;                 // [slices][seq_q][D] FP32, zero on entry (accumulated by reductions)
    float* dk;                 // [slices][seq_k][D] FP32
    float* dv;                 // [slices][seq_k][D] FP32
    unsigned long long timeout_ns;
    int causal;                // 1: query i sees keys j <= i + causal_off only
    int causal_off;            // seq_k - seq_q
};

// Work item r of this CTA: (slice, key tile) and its query tiles
// [q_begin, nq_tiles).  With the causal mask a key tile is seen only by the
// queries at or after its first key (minus the offset), so low key tiles have
// the most steps: items go heaviest first (key-tile-major) and are dealt in a
// snake order, as the forward deals its causal items.
struct BwdItem {
    int slice, kt, q_begin;
    bool valid;
};

__device__ __forceinline__ BwdItem bwd_item(const BwdArgs& a, int r)
{
    const int G = gridDim.x, b = blockIdx.x;
    BwdItem it;
    if (a.causal) {
        const int w = r * G + ((r & 1) ? G - 1 - b : b);
        it.valid = w < a.n_items;
        it.kt = w / a.slices;
        it.slice = w % a.slices;
        const int first_q = it.kt * 128 - a.causal_off;  // first query that sees a key of the tile
        it.q_begin = first_q <= 0 ? 0 : first_q / 64;
    } else {
        const int w = r * G + b;
        it.valid = w < a.n_items;
        it.slice = w / a.nk_tiles;
        it.kt = w % a.nk_tiles;
        it.q_begin = 0;
    }
    return it;
}

__device__ __forceinline__ uint32_t pack_bf162(float lo, float hi)
{
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// kWithhold (test instantiation only, fp4attn_selftest_backward_abort): the
// first gradient thread never makes its first s_free arrival, so the S
// issuer's bounded wait for step 1 runs out and the abort path runs.
template <int D, bool kWithhold = false>
__global__ void __launch_bounds__(512, 1)
    fp4_attention_bwd_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kq,
                             const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_qq,
                             const BwdArgs args)
{
    using C = BwdCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sK = smem + C::OFF_K;
    uint8_t* sKsf = smem + C::OFF_KSF;
    uint8_t* sV = smem + C::OFF_V;
    uint8_t* sKq = smem + C::OFF_KQ;
    uint8_t* sStage = smem + C::OFF_STAGE;
    uint8_t* sDS = smem + C::OFF_DS;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* kv_full = bars;
    uint64_t* kv_empty = bars + 1;             // the item's MMAs are done with K, V, Kq (commit)
    uint64_t* q_full = bars + 2;               // [QST]
    uint64_t* q_empty = q_full + C::QST;       // [QST] MMAs done (commit) + gradient warpgroups done (256)
    uint64_t* s_full = q_empty + C::QST;       // S^T and dP^T computed (commit)
    uint64_t* s_free = s_full + 1;             // S^T and dP^T copied to registers (256)
    uint64_t* ds_full = s_free + 1;            // P in TMEM and dZ in shared memory (256)
    uint64_t* ds_free = ds_full + 1;           // dV, dK, dQ^T MMAs done with P and dZ (commit)
    uint64_t* dq_full = ds_free + 1;           // dQ^T computed (commit)
    uint64_t* dq_free = dq_full + 1;           // dQ^T copied to registers (128)
    uint64_t* acc_full = dq_free + 1;          // the item's dV, dK complete (commit)
    uint64_t* acc_free = acc_full + 1;         // dV, dK copied out (128)
    uint64_t* drain_bar = acc_free + 1;        // the S issuer's MMAs complete (exit)
    uint64_t* drain_bar2 = drain_bar + 1;      // the gradient issuer's MMAs complete (exit)

    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        ptx::mbar_init(kv_full, 1);
        ptx::mbar_init(kv_empty, 1);
        for (int i = 0; i < C::QST; i++) {
            ptx::mbar_init(&q_full[i], 1);
            ptx::mbar_init(&q_empty[i], 1 + 256);
        }
        ptx::mbar_init(s_full, 1);
        ptx::mbar_init(s_free, 256);
        ptx::mbar_init(ds_full, 256);
        ptx::mbar_init(ds_free, 1);
        ptx::mbar_init(dq_full, 1);
        ptx::mbar_init(dq_free, 128);
        ptx::mbar_init(acc_full, 1);
        ptx::mbar_init(acc_free, 128);
        ptx::mbar_init(drain_bar, 1);
        ptx::mbar_init(drain_bar2, 1);
        abort_sh = 0;
        ptx::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        ptx::prefetch_tmap(&tm_k);
        ptx::prefetch_tmap(&tm_q);
        ptx::prefetch_tmap(&tm_v);
        ptx::prefetch_tmap(&tm_kq);
        ptx::prefetch_tmap(&tm_do);
        ptx::prefetch_tmap(&tm_qq);
    }
    if (warp == 1) {
        ptx::tmem_alloc(&tmem_base_sh, 512);
        ptx::tmem_relinquish();
    }
    if constexpr (C::DCH < C::KQ_CHUNKS) {
        // Kq chunks past head_dim (rows D..127 of the dQ^T MMA's A) are zero.
        constexpr int kPad = (C::KQ_CHUNKS - C::DCH) * C::BK * C::CB / 16;
        for (int u = threadIdx.x; u < kPad; u += blockDim.x)
            *reinterpret_cast<uint4*>(sKq + C::DCH * C::BK * C::CB + 16 * u) = make_uint4(0u, 0u, 0u, 0u);
        ptx::fence_proxy_async_smem();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    const WaitCtx wctx{&abort_sh, args.timeout_ns};
    // The set-up above overlaps the previous grid's tail (programmatic
    // dependent launch); the prepared operands are read from here on.
    ptx::grid_dependency_wait();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int it = 0, g = 0;
            bool ok = true;
            for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
                const BwdItem item = bwd_item(args, r);
                if (!item.valid || item.q_begin >= args.nq_tiles) continue;
                if (it > 0 && !wait_phase(kv_empty, (it - 1) & 1, wctx, kSiteKEmpty)) break;
                ptx::mbar_arrive_expect_tx(kv_full, C::KV_TX);
                ptx::tma_load_3d(sK, &tm_k, kv_full, 0, item.kt * C::BK, item.slice);
                ptx::bulk_load(sKsf, args.k_sf + (static_cast<size_t>(item.slice) * args.nk_tiles + item.kt) * C::SF_BYTES,
                               C::SF_BYTES, kv_full);
#pragma unroll
                for (int c = 0; c < C::DCH; c++) {
                    ptx::tma_load_3d(sV + c * C::BK * C::CB, &tm_v, kv_full, C::CHE * c, item.kt * C::BK, item.slice);
                    ptx::tma_load_3d(sKq + c * C::BK * C::CB, &tm_kq, kv_full, C::CHE * c, item.kt * C::BK, item.slice);
                }
                it++;
                for (int qi = item.q_begin; qi < args.nq_tiles; qi++, g++) {
                    const int qs = g % C::QST;
                    if (g >= C::QST && !wait_phase(&q_empty[qs], ((g / C::QST) - 1) & 1, wctx, kSiteQEmpty)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = sStage + qs * C::STAGE_BYTES;
                    ptx::mbar_arrive_expect_tx(&q_full[qs], C::STAGE_TX);
                    ptx::tma_load_3d(st + C::SQ_Q, &tm_q, &q_full[qs], 0, qi * C::BQ, item.slice);
                    ptx::bulk_load(st + C::SQ_QSF,
                                   args.q_sf + (static_cast<size_t>(item.slice) * args.nq_tiles + qi) * C::SF_BYTES,
                                   C::SF_BYTES, &q_full[qs]);
#pragma unroll
                    for (int c = 0; c < C::DCH; c++) {
                        ptx::tma_load_3d(st + C::SQ_DO + c * C::BQ * C::CB, &tm_do, &q_full[qs], C::CHE * c,
                                         qi * C::BQ, item.slice);
                        ptx::tma_load_3d(st + C::SQ_QQ + c * C::BQ * C::CB, &tm_qq, &q_full[qs], C::CHE * c,
                                         qi * C::BQ, item.slice);
                    }
                    const size_t row = static_cast<size_t>(item.slice) * args.sq_pad + qi * C::BQ;
                    ptx::bulk_load(st + C::SQ_LSE, args.nlse2 + row, C::BQ * 4, &q_full[qs]);
                    ptx::bulk_load(st + C::SQ_DD, args.ndd + row, C::BQ * 4, &q_full[qs]);
                }
            }
            // Every copy this thread issued lands before the CTA exits.
            const unsigned long long drain_ns = 2ull * args.timeout_ns;
            if (it > 0) drain_phase(kv_full, (it - 1) & 1, drain_ns);
            for (int i = g - C::QST < 0 ? 0 : g - C::QST; i < g; i++)
                drain_phase(&q_full[i % C::QST], (i / C::QST) & 1, drain_ns);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ S issuer
        if (lane == 0) {
            constexpr uint32_t qk_layout = ptx::swizzle_mode_for_bytes(C::QK_ROW);
            const uint64_t kdesc0 = ptx::make_sdesc(ptx::smem_u32(sK), 16, 8 * C::QK_ROW, qk_layout);
            const uint64_t ksfdesc = ptx::make_sdesc(ptx::smem_u32(sKsf), 0, 128, ptx::kSwizzleNone);
            constexpr uint32_t idesc_dp = ptx::idesc_f16x(128, C::BQ, 0, false, false);
            int it = 0, g = 0;
            bool ok = true;
            for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
                const BwdItem item = bwd_item(args, r);
                if (!item.valid || item.q_begin >= args.nq_tiles) continue;
                if (!wait_phase(kv_full, it & 1, wctx, kSiteKFull)) break;
                ptx::tc_fence_after();
                // (the previous item's S^T MMAs, which read these columns, were
                // issued before by this thread and run first)
                ptx::tc_cp_32x128b_warpx4(tmem + C::SFA_COL, ksfdesc);
                for (int qi = item.q_begin; qi < args.nq_tiles; qi++, g++) {
                    // S^T and dP^T of step g (stage g % QST) into their TMEM columns,
                    // once step g-1's are in the gradient warpgroups' registers.
                    const int qs = g % C::QST;
                    if (!wait_phase(&q_full[qs], (g / C::QST) & 1, wctx, kSiteQFull)) { ok = false; break; }
                    if (g > 0 && !wait_phase(s_free, (g - 1) & 1, wctx, kSiteSFree)) { ok = false; break; }
                    ptx::tc_fence_after();
                    uint8_t* st = sStage + qs * C::STAGE_BYTES;
                    const uint32_t sfb = tmem + C::SFB_COL;
                    ptx::tc_cp_32x128b_warpx4(sfb, ptx::make_sdesc(ptx::smem_u32(st + C::SQ_QSF), 0, 128, ptx::kSwizzleNone));
                    const uint64_t qdesc = ptx::make_sdesc(ptx::smem_u32(st + C::SQ_Q), 16, 8 * C::QK_ROW, qk_layout);
#pragma unroll
                    for (int kk = 0; kk < C::KSTEPS; kk++) {
                        const uint32_t sf_id = 2u * (kk & 1);
                        ptx::mma_mxf4(tmem + C::S_COL, kdesc0 + static_cast<uint64_t>((kk * 32) >> 4),
                                      qdesc + static_cast<uint64_t>((kk * 32) >> 4),
                                      ptx::idesc_mxf4(128, C::BQ, sf_id, sf_id), (tmem + C::SFA_COL) | (sf_id << 30),
                                      sfb | (sf_id << 30), kk > 0 ? 1u : 0u);
                    }
                    // dP^T = V dO^T: both K-major (K = head_dim), 16 columns per MMA.
#pragma unroll
                    for (int kk = 0; kk < D / 16; kk++) {
                        const uint32_t off = (kk % C::KPC) * 32;  // 16 columns = 32 bytes into the chunk's rows
                        const uint64_t a = ptx::make_sdesc(ptx::smem_u32(sV + (kk / C::KPC) * C::BK * C::CB) + off, 16,
                                                           8 * C::CB, C::CSW);
                        const uint64_t b = ptx::make_sdesc(
                            ptx::smem_u32(st + C::SQ_DO + (kk / C::KPC) * C::BQ * C::CB) + off, 16, 8 * C::CB, C::CSW);
                        ptx::mma_f16_ss(tmem + C::DP_COL, a, b, idesc_dp, kk > 0 ? 1u : 0u);
                    }
                    ptx::tc_commit(s_full);
                }
                it++;
            }
            // Every tcgen05 op this thread issued completes before TMEM is freed.
            ptx::tc_commit(drain_bar);
            drain_phase(drain_bar, 0, 2ull * args.timeout_ns);
        }
        __syncwarp();
    } else if (warp == 2) {
        // ------------------------------------------------------------ gradient issuer
        // Its operands: P (TMEM) and dZ (shared memory) from the gradient
        // warpgroups (ds_full), dO and Qq from the query stage, Kq from the
        // item's tiles.  The stage and the item's tiles are waited for here as
        // well, so that their copies are seen complete by this thread.
        if (lane == 0) {
            constexpr uint32_t idesc_dv = ptx::idesc_f16x(128, D, 0, false, true);
            constexpr uint32_t idesc_dk = ptx::idesc_f16x(128, D, 1, false, true);
            constexpr uint32_t idesc_dq = ptx::idesc_f16x(128, C::BQ, 1, true, true);
            const uint32_t sw128 = ptx::kSwizzle128B;
            int it = 0, g = 0;
            bool ok = true;
            for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
                const BwdItem item = bwd_item(args, r);
                if (!item.valid || item.q_begin >= args.nq_tiles) continue;
                if (!wait_phase(kv_full, it & 1, wctx, kSiteKFull)) break;
                for (int qi = item.q_begin; qi < args.nq_tiles; qi++, g++) {
                    const int qs = g % C::QST;
                    uint8_t* st = sStage + qs * C::STAGE_BYTES;
                    if (!wait_phase(&q_full[qs], (g / C::QST) & 1, wctx, kSiteQFull)) { ok = false; break; }
                    if (!wait_phase(ds_full, g & 1, wctx, kSitePFull)) { ok = false; break; }
                    if (qi == item.q_begin && it > 0 && !wait_phase(acc_free, (it - 1) & 1, wctx, kSitePvDone)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    // dV += P^T dO (P from TMEM: lanes = keys, columns = queries),
                    // dK += dZ^T Qq (dZ K-major in shared memory); B MN-major
                    // (N = head_dim in CHE-column chunks, K = queries).
#pragma unroll
                    for (int kk = 0; kk < C::BQ / 16; kk++) {
                        const uint64_t ad = ptx::make_sdesc(ptx::smem_u32(sDS) + kk * 32, 16, 1024, sw128);
                        const uint64_t bo = ptx::make_sdesc(ptx::smem_u32(st + C::SQ_DO) + kk * 16 * C::CB,
                                                            C::BQ * C::CB, 8 * C::CB, C::CSW);
                        const uint64_t bq = ptx::make_sdesc(ptx::smem_u32(st + C::SQ_QQ) + kk * 16 * C::CB,
                                                            C::BQ * C::CB, 8 * C::CB, C::CSW);
                        const uint32_t acc = (qi > item.q_begin || kk > 0) ? 1u : 0u;
                        ptx::mma_f16_ts(tmem + C::DV_COL, tmem + C::P_COL + kk * 8, bo, idesc_dv, acc);
                        ptx::mma_f16_ss(tmem + C::DK_COL, ad, bq, idesc_dk, acc);
                    }
                    if (g > 0 && !wait_phase(dq_free, (g - 1) & 1, wctx, kSiteSFree)) { ok = false; break; }
                    ptx::tc_fence_after();
                    // dQ^T = Kq^T dZ^T: A MN-major (M = head_dim in CHE-row chunks, K = keys),
                    // B MN-major (N = queries, K = keys).
#pragma unroll
                    for (int kk = 0; kk < C::BK / 16; kk++) {
                        const uint64_t a = ptx::make_sdesc(ptx::smem_u32(sKq) + kk * 16 * C::CB, C::BK * C::CB, 8 * C::CB,
                                                           C::CSW);
                        const uint64_t b = ptx::make_sdesc(ptx::smem_u32(sDS) + kk * 16 * 128, C::BK * 128, 1024, sw128);
                        ptx::mma_f16_ss(tmem + C::DQ_COL, a, b, idesc_dq, kk > 0 ? 1u : 0u);
                    }
                    ptx::tc_commit(ds_free);
                    ptx::tc_commit(dq_full);
                    // (step g's S^T and dP^T, the stage's other readers, completed
                    // before its gradient warpgroups stored P and dZ)
                    ptx::tc_commit(&q_empty[qs]);
                }
                if (!ok) break;
                // Every MMA of the item has been issued: this thread's dV, dK and
                // dQ^T last, after the S issuer's (whose completion the gradient
                // warpgroups saw before storing the last P and dZ).
                ptx::tc_commit(acc_full);
                ptx::tc_commit(kv_empty);
                it++;
            }
            ptx::tc_commit(drain_bar2);
            drain_phase(drain_bar2, 0, 2ull * args.timeout_ns);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------------ gradient warpgroups
        const int h = (warp - 4) / 4;              // queries [32h, 32h + 32) of each step
        const int kr = (warp % 4) * 32 + lane;     // key row of the item = TMEM lane
        const uint32_t lane_off = static_cast<uint32_t>((warp % 4) * 32) << 16;
        const float c = args.scale_log2, sc = args.scale;
        int g = 0;
        bool ok = true;
        for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
            const BwdItem item = bwd_item(args, r);
            if (!item.valid || item.q_begin >= args.nq_tiles) continue;
            const int key = item.kt * C::BK + kr;
            const bool key_ok = key < args.seq_k;
            // Query q sees this key iff q >= lim.
            const int lim = args.causal ? key - args.causal_off : INT_MIN;
            for (int qi = item.q_begin; qi < args.nq_tiles; qi++, g++) {
                const int qs = g % C::QST;
                if (!__all_sync(0xffffffffu, wait_phase(s_full, g & 1, wctx, kSiteSFull))) { ok = false; break; }
                ptx::tc_fence_after();
                uint32_t sr[32], dr[32];
                ptx::tmem_ld32(tmem + lane_off + C::S_COL + 32 * h, sr);
                ptx::tmem_ld32(tmem + lane_off + C::DP_COL + 32 * h, dr);
                ptx::tc_wait_ld();
                ptx::tc_fence_before();
                if (!kWithhold || threadIdx.x != 128 || g != 0) ptx::mbar_arrive(s_free);
                // -lse2 and -Dd of this stage (the TMA's writes are visible after the wait).
                if (!__all_sync(0xffffffffu, wait_phase(&q_full[qs], (g / C::QST) & 1, wctx, kSiteQFull))) {
                    ok = false;
                    break;
                }
                const uint8_t* st = sStage + qs * C::STAGE_BYTES;
                // -lse2 and -Dd of this warpgroup's 32 queries (4 per float4).
                const float4* nl4 = reinterpret_cast<const float4*>(st + C::SQ_LSE) + 8 * h;
                const float4* nd4 = reinterpret_cast<const float4*>(st + C::SQ_DD) + 8 * h;
                const int q0 = qi * C::BQ + 32 * h;
                // P = 2^(S c - lse2) and dZ = (P scale) (dP - Dd), two queries
                // per packed FP32x2 operation.  Every query of this warp's slice
                // of the step sees every key of the warp (no mask work), or not.
                const bool full = __all_sync(0xffffffffu, key_ok && q0 >= lim);
                uint32_t pk[16], dk[16];
                if (full) {
#pragma unroll
                    for (int c4 = 0; c4 < 8; c4++) {
                        const float4 L = nl4[c4], Dv = nd4[c4];
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int q = 4 * c4 + 2 * e;
                            const float2 x = ptx::ffma2(make_float2(__uint_as_float(sr[q]), __uint_as_float(sr[q + 1])),
                                                        make_float2(c, c),
                                                        e ? make_float2(L.z, L.w) : make_float2(L.x, L.y));
                            const float2 pr = make_float2(ptx::ex2_approx(x.x), ptx::ex2_approx(x.y));
                            const float2 t = ptx::fadd2(make_float2(__uint_as_float(dr[q]), __uint_as_float(dr[q + 1])),
                                                        e ? make_float2(Dv.z, Dv.w) : make_float2(Dv.x, Dv.y));
                            const float2 z = ptx::fmul2(ptx::fmul2(pr, make_float2(sc, sc)), t);
                            pk[q / 2] = ptx::pack_half2(pr.x, pr.y);
                            dk[q / 2] = pack_bf162(z.x, z.y);
                        }
                    }
                } else {
#pragma unroll
                    for (int c4 = 0; c4 < 8; c4++) {
                        const float4 L = nl4[c4], Dv = nd4[c4];
                        const float Ls[4] = {L.x, L.y, L.z, L.w}, Ds[4] = {Dv.x, Dv.y, Dv.z, Dv.w};
                        float pv[4], zv[4];
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int q = 4 * c4 + e;
                            float pr = ptx::ex2_approx(fmaf(__uint_as_float(sr[q]), c, Ls[e]));
                            if (!key_ok || q0 + q < lim) pr = 0.f;
                            pv[e] = pr;
                            zv[e] = (pr * sc) * (__uint_as_float(dr[q]) + Ds[e]);
                        }
                        pk[2 * c4] = ptx::pack_half2(pv[0], pv[1]);
                        pk[2 * c4 + 1] = ptx::pack_half2(pv[2], pv[3]);
                        dk[2 * c4] = pack_bf162(zv[0], zv[1]);
                        dk[2 * c4 + 1] = pack_bf162(zv[2], zv[3]);
                    }
                }
                // The previous step's dV, dK and dQ^T MMAs must be done reading P and dZ.
                if (g > 0 && !__all_sync(0xffffffffu, wait_phase(ds_free, (g - 1) & 1, wctx, kSitePvDone))) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                ptx::tmem_st16(tmem + lane_off + C::P_COL + 16 * h, pk);
                // dZ row kr: 128 bytes, 16-byte unit u at (u ^ (kr & 7)) (128-byte
                // swizzle); this warpgroup's queries are units 4h .. 4h + 3.
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int pu = (4 * h + u) ^ (kr & 7);
                    *reinterpret_cast<uint4*>(sDS + kr * 128 + pu * 16) =
                        make_uint4(dk[4 * u], dk[4 * u + 1], dk[4 * u + 2], dk[4 * u + 3]);
                }
                ptx::fence_proxy_async_smem();
                ptx::tc_wait_st();
                ptx::tc_fence_before();
                ptx::mbar_arrive(ds_full);
                ptx::mbar_arrive(&q_empty[qs]);
            }
        }
    } else if (warp >= 12) {
        // ------------------------------------------------------------ dQ warpgroup
        const int wq = warp - 12;
        const int tr = wq * 32 + lane;             // TMEM lane: head-dim row of dQ^T, key row of dV / dK
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        int g = 0, it = 0;
        bool ok = true;
        for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
            const BwdItem item = bwd_item(args, r);
            if (!item.valid) continue;
            const int key = item.kt * C::BK + tr;
            const size_t orow = (static_cast<size_t>(item.slice) * args.seq_k + key) * D;
            if (item.q_begin >= args.nq_tiles) {
                // No query sees these keys: dK = dV = 0.
                if (key < args.seq_k)
                    for (int k = 0; k < D; k += 4) {
                        *reinterpret_cast<float4*>(args.dv + orow + k) = make_float4(0.f, 0.f, 0.f, 0.f);
                        *reinterpret_cast<float4*>(args.dk + orow + k) = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                continue;
            }
            for (int qi = item.q_begin; qi < args.nq_tiles; qi++, g++) {
                if (!__all_sync(0xffffffffu, wait_phase(dq_full, g & 1, wctx, kSiteSFull))) { ok = false; break; }
                ptx::tc_fence_after();
                uint32_t v[2][32];
                ptx::tmem_ld32(tmem + lane_off + C::DQ_COL, v[0]);
                ptx::tmem_ld32(tmem + lane_off + C::DQ_COL + 32, v[1]);
                ptx::tc_wait_ld();
                ptx::tc_fence_before();
                ptx::mbar_arrive(dq_free);
                if (tr < D) {  // (rows past head_dim are the zero Kq chunks' products)
                    // Query row q0 + j of dQ gets column tr of the tile: the warp's
                    // 32 lanes add 32 consecutive floats of that row.
                    const int q0 = qi * C::BQ;
                    const int nrow = min(C::BQ, args.seq_q - q0);
                    float* dst = args.dq + (static_cast<size_t>(item.slice) * args.seq_q + q0) * D + tr;
#pragma unroll
                    for (int j = 0; j < 64; j++) {
                        if (j < nrow) atomicAdd(dst + static_cast<size_t>(j) * D, __uint_as_float(v[j / 32][j % 32]));
                    }
                }
            }
            if (!ok) break;
            // dV and dK of the item: thread = key row.
            if (!__all_sync(0xffffffffu, wait_phase(acc_full, it & 1, wctx, kSitePvDone))) break;
            ptx::tc_fence_after();
#pragma unroll 1
            for (int k = 0; k < D / 32; k++) {
                uint32_t a[32], b[32];
                ptx::tmem_ld32(tmem + lane_off + C::DV_COL + 32 * k, a);
                ptx::tmem_ld32(tmem + lane_off + C::DK_COL + 32 * k, b);
                ptx::tc_wait_ld();
                if (key < args.seq_k) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        *reinterpret_cast<float4*>(args.dv + orow + 32 * k + i) =
                            make_float4(__uint_as_float(a[i]), __uint_as_float(a[i + 1]), __uint_as_float(a[i + 2]),
                                        __uint_as_float(a[i + 3]));
                        *reinterpret_cast<float4*>(args.dk + orow + 32 * k + i) =
                            make_float4(__uint_as_float(b[i]), __uint_as_float(b[i + 1]), __uint_as_float(b[i + 2]),
                                        __uint_as_float(b[i + 3]));
                    }
                }
            }
            ptx::tc_fence_before();
            ptx::mbar_arrive(acc_free);
            it++;
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------- prepare
// Q (blockIdx.z == 0, 64-row scale tiles) and K (z == 1, 128-row scale
// tiles) quantised exactly as the forward's pre-pass does (codes, scale
// tiles with scale 127 on padding rows), plus the dequantised values -- the
// numbers the forward's MMA multiplied -- as BF16 (exact: 3 significant bits
// and an exponent inside BF16's range; FP32 input whose block maximum reaches
// 2^126 would saturate).  One lane per block of 32 elements.
struct BwdQuantJob {
    const void* x;          // [slices][seq][D] of InT
    uint8_t* codes;         // [slices][seq][DP/2] (blocks past D zero)
    uint8_t* sf;            // [slices][ntiles][512]
    __nv_bfloat16* deq;     // [slices][seq][D]
    int seq, tile_rows, tile_shift, ntiles;
};

template <typename InT, int D>
__global__ void __launch_bounds__(256) bwd_quantize_kernel(const BwdQuantJob jq, const BwdQuantJob jk, int ocp_mode)
{
    const BwdQuantJob& j = blockIdx.z == 0 ? jq : jk;
    constexpr int DP = (D + 63) / 64 * 64;
    constexpr int kNB = DP / 32;  // blocks of 32 per code row (those past D: zero codes, scale 127)
    const int64_t slice = blockIdx.y;
    const int total = j.ntiles * j.tile_rows * kNB;
    const InT* xs = static_cast<const InT*>(j.x) + slice * j.seq * D;
    uint8_t* cs = j.codes + slice * j.seq * (DP / 2);
    uint8_t* fs = j.sf + slice * j.ntiles * 512;
    __nv_bfloat16* ds = j.deq + slice * j.seq * D;
    // Twice the E2M1 magnitude of code bits 0-2 (0, 1, 2, 3, 4, 6, 8, 12), one
    // nibble each; bit 3 of a code is the sign.
    constexpr uint32_t kMag2 = 0xC8643210u;
    auto mag = [](uint32_t n) { return static_cast<float>((kMag2 >> (4u * (n & 7u))) & 15u) * 0.5f; };
    for (int blk = blockIdx.x * blockDim.x + threadIdx.x; blk < total; blk += gridDim.x * blockDim.x) {
        const int b = blk % kNB, r = blk / kNB;
        uint32_t sb = 127u;
        if (r < j.seq && b * 32 >= D) {
            *reinterpret_cast<uint4*>(cs + static_cast<int64_t>(r) * (DP / 2) + b * 16) = make_uint4(0u, 0u, 0u, 0u);
        } else if (r < j.seq) {
            uint4 packed;
            sb = quantize32<InT>(xs + static_cast<int64_t>(r) * D + b * 32, ocp_mode, packed);
            if (sb == 255u) sb = 254u;  // as the forward stores it (codes are all zero then)
            *reinterpret_cast<uint4*>(cs + static_cast<int64_t>(r) * (DP / 2) + b * 16) = packed;
            // 2^(sb - 127) exactly (sb 0 is the subnormal 2^-127).
            const float sc = sb ? __uint_as_float(sb << 23) : __uint_as_float(1u << 22);
            const uint32_t w[4] = {packed.x, packed.y, packed.z, packed.w};
            uint32_t o[16];
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    const uint32_t n0 = (w[k] >> (4 * i)) & 15u, n1 = (w[k] >> (4 * i + 4)) & 15u;
                    const float v0 = (n0 & 8u ? -mag(n0) : mag(n0)) * sc;
                    const float v1 = (n1 & 8u ? -mag(n1) : mag(n1)) * sc;
                    o[4 * k + i / 2] = pack_bf162(v0, v1);
                }
            uint4* dst = reinterpret_cast<uint4*>(ds + static_cast<int64_t>(r) * D + b * 32);
#pragma unroll
            for (int k = 0; k < 4; k++) dst[k] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
        }
        const int tile = r >> j.tile_shift, rr = r & (j.tile_rows - 1);
        fs[static_cast<int64_t>(tile) * 512 + sf_tile_offset(j.tile_rows, rr, b)] = static_cast<uint8_t>(sb);
    }
}

// FP32 input: V and dO rounded to the FP16 copies the kernel's MMAs read
// (V as the forward rounds it).  Job blockIdx.y, n4 float4 each.
struct BwdConvJob {
    const float4* src;
    uint2* dst;
    int64_t n4;
};

__global__ void __launch_bounds__(256) bwd_convert_kernel(const BwdConvJob jv, const BwdConvJob jo)
{
    const BwdConvJob& j = blockIdx.y == 0 ? jv : jo;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < j.n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 f = j.src[i];
        __half2 a = __floats2half2_rn(f.x, f.y), b = __floats2half2_rn(f.z, f.w);
        j.dst[i] = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    }
}

// E consecutive elements of T at p as floats, with one vector load when E
// elements span 4, 8 or 16 bytes (p is then aligned to that span).
template <typename T, int E>
__device__ __forceinline__ void load_floats(const T* __restrict__ p, float (&v)[E])
{
    constexpr int kBytes = E * static_cast<int>(sizeof(T));
    if constexpr (kBytes == 16 || kBytes == 8 || kBytes == 4) {
        using V = std::conditional_t<kBytes == 16, uint4, std::conditional_t<kBytes == 8, uint2, uint32_t>>;
        const V raw = *reinterpret_cast<const V*>(p);
        const T* t = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int e = 0; e < E; e++) {
            if constexpr (sizeof(T) == 4) v[e] = t[e];
            else v[e] = __half2float(t[e]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < E; e++) {
            if constexpr (sizeof(T) == 4) v[e] = p[e];
            else v[e] = __half2float(p[e]);
        }
    }
}

// Per query row, negated for the kernel's fused adds: -Dd with Dd = sum_c
// dO_c O_c (FP32, dO as the FP16 value the MMAs read) and -lse2 with lse2 =
// lse * log2(e); padding rows up to sq_pad get 0 and -inf (their
// probabilities are 0).  One warp per row, D / 32 elements per lane.
template <int D, typename OT, typename IT>
__global__ void __launch_bounds__(256) bwd_rows_kernel(const IT* __restrict__ dout, const OT* __restrict__ out,
                                                        const float* __restrict__ lse, float* __restrict__ nlse2,
                                                        float* __restrict__ ndd, int seq_q, int sq_pad)
{
    const int row = blockIdx.x * 8 + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (row >= sq_pad) return;
    const int64_t slice = blockIdx.y;
    const int64_t o = slice * sq_pad + row;
    if (row >= seq_q) {
        if (lane == 0) {
            ndd[o] = 0.f;
            nlse2[o] = -INFINITY;
        }
        return;
    }
    const int64_t base = (slice * seq_q + row) * D;
    // Lane l takes the D/32 consecutive elements starting at l * D/32 (one
    // contiguous transaction per warp and tensor).
    constexpr int E = D / 32;
    float gv[E], ov[E];
    const int64_t at = base + lane * E;
    load_floats<IT, E>(dout + at, gv);
    load_floats<OT, E>(out + at, ov);
    if constexpr (sizeof(IT) == 4) {
#pragma unroll
        for (int e = 0; e < E; e++) gv[e] = __half2float(__float2half_rn(gv[e]));
    }
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < E; e++) acc = fmaf(gv[e], ov[e], acc);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if (lane == 0) {
        ndd[o] = -acc;
        nlse2[o] = lse[slice * seq_q + row] * -1.4426950408889634f;
    }
}

}  // namespace fp4attn
