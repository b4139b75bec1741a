// attention_pair.cuh -- FP4 fused attention forward, two query tiles per CTA,
// for head_dim <= 128 on sm_100a.
//
// Same computation as fp4_attention_fwd_kernel (attention.cuh) -- the
// reference kernel fused_fp4_attention (common.h:68-328) with Q, K in
// E2M1 + UE8M0 and V, P in FP16 -- with a different division of the work.
// A work item is 256 query rows of one (batch, head) slice, as two
// independent 128-row tiles T0, T1, whose keys are walked in 64-row tiles.
// The kernel is persistent: one CTA per SM takes items in rounds of gridDim.x
// (pair_item: without a mask consecutive items share a slice's K/V in L2),
// and every barrier phase and ring index runs on across items, so the next
// item's Q, K, V and first S are fetched and computed while the current
// item's last step and epilogue run.  Roles:
//
//   warp 0      TMA producer: per item both Q tiles (once the previous item's
//               S MMAs are done with them), then K (codes + scale tile) and V
//               tiles through KST/VST-stage mbarrier rings.
//   warp 1      S issuer: S_t = Q_t K_j^T (tcgen05.mma kind::mxf4 block_scale,
//               M128 N64) for t = 0, 1; S_t for step j+1 is issued as soon
//               as softmax warpgroup t has copied S_t of step j to registers.
//   warp 2      P.V issuer: O_t += P_t [V_j | 1] (tcgen05.mma kind::f16, P read
//               from TMEM) as soon as softmax warpgroup t has stored P_t.  Each
//               V stage carries, after V's own swizzled chunks, one constant
//               chunk whose first 16 columns are 1.0, and the MMA runs 16
//               columns wider than V: O_t's extra columns accumulate the row
//               sum l = sum_j rowsum(P_t) on the tensor core (from the same
//               FP16 P that multiplies V), rescaled together with O.
//   warp 3      idle (completes the control warpgroup for setmaxnreg)
//   warps 4-7   softmax of tile T0; warps 8-11 softmax of tile T1.  Thread =
//               query row = TMEM lane; each thread owns its whole 64-column S
//               row, so the row max, the exponentials, the row sum, the lazy O
//               rescale and the final O / l need no exchange between warps.
//               The exponentials of a step are computed against the running
//               reference max while the step's row max is formed alongside
//               (kSpec); only when a row max jumps past the lazy-rescale
//               threshold is the step redone max-first, so the max is off the
//               critical path.
//
// Small problems (kSmall, a separate instantiation so that the kernel for
// large problems keeps its own code).  With seq_q <= 128 an item is one query
// tile (qtiles = 1: tile T1 and its warpgroup stay idle instead of computing
// padding rows), and when there are fewer (slice, query tile group) groups
// than SMs the keys of a group are split into kparts partitions, one work item
// each (flash-decoding): the item writes its unnormalised O, row max and row
// sum to the workspace, and the CTA whose item completes a group last (a
// per-group arrival counter) merges the partitions into the output.
//
// TMEM columns (512 allocated): S_0 [0,64), S_1 [64,128), O_0, O_1 (NPV each:
// V's padded width + 16 columns holding l), P_0, P_1 (32 each: 64 FP16
// pairs), the two Q scale column groups, then KST groups of K scale columns.
//
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records
// FP4ATTN_ETIMEOUT, all roles leave their loops, in-flight copies and MMAs are
// drained (bounded), TMEM is freed and the CTA returns.  Nothing traps.
#pragma once

#include <type_traits>

#include "attention.cuh"
#include "quantize.cuh"

namespace fp4attn {

// Most key partitions per query group (the planner caps kparts at this).
constexpr int kMaxKParts = 16;

// QB: Q buffers (2 tiles each).  The kernel that quantises Q itself
// (kFuseQ) writes item i+1's Q into one buffer while item i reads the other.
template <int D, int QB = 1>
struct PairCfg {
    static constexpr int BM = 128;                          // rows per query tile (MMA M)
    static constexpr int BN = 64;                           // keys per step
    static constexpr int DP = (D + 63) / 64 * 64;           // head_dim padded to the MMA K step
    static constexpr int QK_ROW = DP / 2;                   // bytes per packed code row
    static constexpr int CW = QK_ROW;                       // swizzle chunk = whole row (32 or 64 B)
    static constexpr int KSTEPS = DP / 64;                  // mxf4 MMAs per S tile
    // Swizzle chunk of a V row (bytes): 128 where it divides the row, else 64
    // (head_dim 32 and 96), so no chunk carries padding columns into P.V.
    static constexpr int VCW = (2 * D) % 128 == 0 ? 128 : 64;
    static constexpr int VCH = (2 * D + VCW - 1) / VCW;     // V chunks (TMA boxes) per tile
    static constexpr int L_COL = VCH * VCW / 2;             // O column holding the row sum l
    static constexpr int NPV = L_COL + 16;                  // P.V MMA width: V chunks + the ones block
    static constexpr int KST = 4;
    static constexpr int VST = 4;
    static_assert(D % 32 == 0 && D <= 128, "the paired kernel covers head_dim <= 128");
    // TMEM
    static constexpr int S_COL = 0;                         // + t * BN
    static constexpr int O_COL = 2 * BN;                    // + t * NPV
    static constexpr int P_COL = O_COL + 2 * NPV;           // + t * BN / 2
    static constexpr int SFA_COL = P_COL + BN;              // + t * 4
    static constexpr int SFB_COL = SFA_COL + 8;             // + stage * 4
    static constexpr int TMEM_USED = SFB_COL + 4 * KST;
    static_assert(TMEM_USED <= 512, "TMEM budget exceeded");
    // shared memory (offsets from a 1024-aligned base)
    static constexpr int align1k(int x) { return (x + 1023) / 1024 * 1024; }
    static constexpr int Q_BYTES = BM * QK_ROW;             // one query tile
    static constexpr int K_BYTES = BN * QK_ROW;
    static constexpr int SF_BYTES = 512;                    // one scale atom (Q: 128 rows x 4, K: 64 rows x 8)
    static constexpr int V_BYTES = VCH * BN * VCW;          // loaded by TMA; the ones chunk follows
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_QSF = align1k(OFF_Q + QB * 2 * Q_BYTES);
    static constexpr int OFF_K = align1k(OFF_QSF + QB * 2 * SF_BYTES);
    static constexpr int K_STRIDE = align1k(K_BYTES);
    static constexpr int OFF_KSF = OFF_K + KST * K_STRIDE;
    static constexpr int OFF_V = align1k(OFF_KSF + KST * SF_BYTES);
    static constexpr int V_STRIDE = align1k(V_BYTES + BN * VCW);
    // Output staging: per softmax warp two buffers of 32 rows x 32 columns
    // (sized for FP32), written swizzled and sent out by TMA stores.
    static constexpr int OST_BYTES = 32 * 32 * 4;
    static constexpr int OFF_OST = OFF_V + VST * V_STRIDE;
    static constexpr int OFF_BAR = OFF_OST + 8 * 2 * OST_BYTES;
    // q_full, q_empty, K ring, V ring, s_full[2], s_free[2], p_full[2], pv_done[2], drain,
    // part_done, merge_go, q_full / q_empty of the second Q buffer, q_first
    static constexpr int NUM_BARS = 2 + 2 * KST + 2 * VST + 8 + 1 + 2 + 3;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 1024;  // +1024 for base alignment
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget exceeded");
};

struct PairArgs {
    int seq_q, seq_k;
    int nk_tiles;
    int n_pairs;               // query groups (pairs, or single tiles when qtiles == 1) per slice
    int n_items;               // work items = slices * n_pairs * kparts
    int q_sf_tiles;            // 128-row scale tiles per slice in q_sf (even)
    float scale_log2;          // softmax_scale * log2(e)
    void* out;                 // [slices, seq_q, D]
    const uint8_t* q_sf;       // [slices][q_sf_tiles][512]
    const uint8_t* k_sf;       // [slices][nk_tiles][512]
    unsigned long long timeout_ns;
    int causal;                // 1: query i sees keys j <= i + causal_off only
    int causal_off;            // seq_k - seq_q (bottom-right alignment)
    // Small problems (the kSmall kernel; 2, 1, nk_tiles and unused otherwise).
    int qtiles;                // query tiles per item: 2 (a pair) or 1 (seq_q <= 128)
    int kparts;                // key partitions per group (1: the whole key range; no mask)
    int nk_part;               // key tiles per partition (the last may have fewer)
    // kparts > 1: per (item, tile) 128 rows of (reference max m in log2 units,
    // row sum l) and, written through tm_p, of unnormalised FP32 O; one
    // arrival counter per group, zero between launches.
    float2* part_ml;           // [n_items][qtiles][128]
    const float* part_o;       // [n_items][qtiles][128][D]
    unsigned* part_count;      // [slices * n_pairs]
    // kFuseQ: FP16 Q [slices][seq_q][D], quantised by the kernel itself, and
    // the scale rule (1: the OCP "/6" rule).
    const __half* q_in;
    int ocp_mode;
    // kLse: per query row ln(sum_j exp(scale * S_ij)) -- the row's reference
    // max and row sum as one number -- for the backward pass, [slices][seq_q].
    // A row that sees no key gets +inf (its probabilities are all zero).
    float* lse;
};

// ln(2): the log-sum-exp leaves the kernel in natural-log units.
constexpr float kLn2 = 0.693147180559945309f;

// Work item r of this CTA's static schedule: (slice, query-tile pair) and its
// number of 64-key steps.  Without a mask items go in slice order (a slice's
// K/V stay in L2 while its pairs run).  With the causal mask an item needs
// keys only up to its last query row, so items go heaviest first (pair-major,
// last pairs first) and are dealt to the CTAs in a snake order (forward on
// even rounds, backward on odd ones), which evens out each CTA's total.
struct PairItem {
    int slice, pair, nk;
    bool valid;
    int k0;                    // kSmall: first key tile of the item's partition
    int idx;                   // kSmall: item index (partial buffers)
};

template <bool kSmall>
__device__ __forceinline__ PairItem pair_item(const PairArgs& a, int r)
{
    const int G = gridDim.x, b = blockIdx.x;
    PairItem it;
    if (a.causal) {
        // (With the mask kparts == 1; with qtiles == 1 a slice has one group, pair 0.)
        const int w = r * G + ((r & 1) ? G - 1 - b : b);
        const int slices = a.n_items / a.n_pairs;
        it.valid = w < a.n_items;
        it.slice = w % slices;
        it.pair = a.n_pairs - 1 - w / slices;
        const int last_row = min(it.pair * 256 + 255, a.seq_q - 1);
        const int hi = last_row + a.causal_off;  // last key any row of the item sees
        it.nk = hi < 0 ? 1 : min(a.nk_tiles, hi / 64 + 1);
        it.k0 = 0;
        it.idx = w;
    } else if constexpr (kSmall) {
        // Consecutive items: the key partitions of one group, then the next
        // group of the same slice (the slice's K/V stay in L2).
        const int w = r * G + b;
        it.valid = w < a.n_items;
        const int grp = w / a.kparts, part = w - grp * a.kparts;
        it.slice = grp / a.n_pairs;
        it.pair = grp - it.slice * a.n_pairs;
        it.k0 = part * a.nk_part;
        it.nk = min(a.nk_tiles - it.k0, a.nk_part);
        it.idx = w;
    } else {
        const int w = r * G + b;
        it.valid = w < a.n_items;
        it.slice = w / a.n_pairs;
        it.pair = w % a.n_pairs;
        it.nk = a.nk_tiles;
    }
    return it;
}

// Register split of the pair kernel.  Its control warpgroup needs fewer
// registers than the one-tile kernel's, so it hands 64 back and the softmax
// warpgroups take 216: 128 x 64 + 256 x 216 = 63,488 <= 384 x 168, and
// 64 + 2 x 216 = 496 registers x 32 lanes per sub-partition.  Measured on the
// 4k x 4k d128 prefill against 80 / 208: 1.1 % faster, d64 1.8 %.  With
// in-kernel Q quantisation warp 3 quantises, which spills at 64 registers, so
// that variant keeps the one-tile kernel's 80 / 208.
template <bool kFuseQ>
struct PairRegs {
    static constexpr int kCtl = kFuseQ ? kCtlRegs : 64;
    static constexpr int kSm = kFuseQ ? kSmRegs : 216;
    static_assert(128 * kCtl + 256 * kSm <= kFwdThreads * kLaunchRegs, "register split exceeds the launch pool");
    static_assert((kCtl + 2 * kSm) * 32 <= 16384, "register split exceeds a sub-partition");
};

// kLse (fp4attn_forward_lse): the epilogue also writes each query row's
// log-sum-exp (args.lse), which the backward pass needs to rebuild the
// normalised probabilities.
// kWithhold (test instantiation only): the first softmax thread never makes
// its first s_free arrival, so the S issuer's bounded wait for step 1 runs out
// and the kernel's own abort path runs: every role leaves its loop, in-flight
// copies and MMAs drain, TMEM is freed and FP4ATTN_ETIMEOUT is recorded.
// kFuseQ: Q is quantised inside the kernel (fp4attn_forward_fused_q), the
// quantiser of the reference kernel (common.h:108-124) moved into this one:
// each CTA's first item is TMA-loaded from the pre-pass as usual (the pre-pass
// quantises just those rows), and the otherwise idle warp 3 quantises every
// later item into the other Q buffer while the current item runs.  The codes and scales are the pre-pass's, bit
// for bit (the same encoder, quantize.cuh), written in the TMA's swizzled
// layout.  Only the large-problem schedule (kSmall false) has this variant.
template <int D, typename OutT, int kPoly8, bool kSpec, bool kSmall = false, bool kWithhold = false,
          bool kFuseQ = false, bool kLse = false>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fp4_attention_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                              const __grid_constant__ CUtensorMap tm_p, const PairArgs args)
{
    static_assert(!(kFuseQ && kSmall), "in-kernel Q quantisation runs the large-problem schedule only");
    using C = PairCfg<D, kFuseQ ? 2 : 1>;
    constexpr int BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + C::OFF_Q;
    uint8_t* sQsf = smem + C::OFF_QSF;
    uint8_t* sK = smem + C::OFF_K;
    uint8_t* sKsf = smem + C::OFF_KSF;
    uint8_t* sV = smem + C::OFF_V;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* q_empty = bars + 1;         // this item's S MMAs are done with Q (tcgen05.commit)
    uint64_t* k_full = bars + 2;
    uint64_t* k_empty = k_full + C::KST;
    uint64_t* v_full = k_empty + C::KST;
    uint64_t* v_empty = v_full + C::VST;
    uint64_t* s_full = v_empty + C::VST;  // [t] S_t computed (tcgen05.commit)
    uint64_t* s_free = s_full + 2;        // [t] S_t copied to registers (128 threads)
    uint64_t* p_full = s_free + 2;        // [t] P_t stored, O_t rescaled (128 threads)
    uint64_t* pv_done = p_full + 2;       // [t] O_t += P_t V complete (tcgen05.commit)
    uint64_t* drain_bar = pv_done + 2;
    uint64_t* part_done = drain_bar + 1;  // kSmall: this item's partials are written (one arrive per softmax warp)
    uint64_t* merge_go = part_done + 1;   // kSmall: the group's arrival count is known (merge_sh)
    // kFuseQ: Q buffer b's barriers (buffer 0 uses q_full / q_empty): qf(b)
    // completes when warp 3 has quantised an item into buffer b, qe(b) when
    // the S MMAs of buffer b's item are done (tcgen05.commit); q_first when the
    // CTA's first item's Q (pre-pass codes) has landed by TMA in buffer 0.
    auto qf = [&](int b) { return b ? merge_go + 1 : q_full; };
    auto qe = [&](int b) { return b ? merge_go + 2 : q_empty; };
    uint64_t* q_first = merge_go + 3;

    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_sh;
    __shared__ int merge_sh;             // kSmall: 1 if this CTA completed the group and merges it

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        ptx::mbar_init(q_full, 1);
        ptx::mbar_init(q_empty, 1);
        for (int i = 0; i < C::KST; i++) {
            ptx::mbar_init(&k_full[i], 1);
            ptx::mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < C::VST; i++) {
            ptx::mbar_init(&v_full[i], 1);
            ptx::mbar_init(&v_empty[i], 1);
        }
        for (int t = 0; t < 2; t++) {
            ptx::mbar_init(&s_full[t], 1);
            ptx::mbar_init(&s_free[t], 128);
            ptx::mbar_init(&p_full[t], 128);
            ptx::mbar_init(&pv_done[t], 1);
        }
        ptx::mbar_init(drain_bar, 2);  // one commit from each MMA issuer
        if constexpr (kSmall) {
            ptx::mbar_init(part_done, 4 * args.qtiles);
            ptx::mbar_init(merge_go, 1);
        }
        if constexpr (kFuseQ) {
            ptx::mbar_init(qf(1), 1);
            ptx::mbar_init(qe(1), 1);
            ptx::mbar_init(q_first, 1);
        }
        abort_sh = 0;
        ptx::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        ptx::prefetch_tmap(&tm_q);
        ptx::prefetch_tmap(&tm_k);
        ptx::prefetch_tmap(&tm_v);
        ptx::prefetch_tmap(&tm_o);
        if (kSmall && args.kparts > 1) ptx::prefetch_tmap(&tm_p);
    }
    if (warp == 1) {
        ptx::tmem_alloc(&tmem_base_sh, 512);
        ptx::tmem_relinquish();
    }
    {
        // The ones chunk of every V stage: logical [BN rows][VCW bytes] FP16,
        // 1.0 in columns 0..15, stored with the stage's swizzle (the 16-byte
        // unit index XORed with address bits 7 and up).
        constexpr uint32_t kMask = C::VCW == 128 ? 7u : C::VCW == 64 ? 3u : 1u;
        constexpr int kUnits = BN * C::VCW / 16;
        for (int u = threadIdx.x; u < C::VST * kUnits; u += blockDim.x) {
            const int stage = u / kUnits, o = (u % kUnits) * 16;
            const int col16 = (o % C::VCW) / 16;  // 16-byte unit within the row: 8 FP16 columns
            const uint32_t phys = static_cast<uint32_t>(o) ^ (((static_cast<uint32_t>(o) >> 7) & kMask) << 4);
            const uint32_t one2 = 0x3C003C00u;    // two FP16 1.0
            const uint4 val = col16 < 2 ? make_uint4(one2, one2, one2, one2) : make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(sV + stage * C::V_STRIDE + C::V_BYTES + phys) = val;
        }
        ptx::fence_proxy_async_smem();
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
    // kFuseQ: quantise the 256 query rows of `item` into Q buffer qb -- units
    // of one 32-element block, unit u = tid, tid + nthr, ... (consecutive
    // threads take consecutive blocks of a row: coalesced 64-byte reads), the
    // next unit's loads in flight while this one is encoded.  Codes go to the
    // swizzled Q tile exactly as the TMA would have placed the pre-pass's
    // codes, scales to the tile's scale atom; rows past seq_q and blocks past
    // head_dim get zero codes and scale 127, as in the pre-pass.
    auto quantize_q = [&](const PairItem& item, int qb, int tid, int nthr) {
        constexpr int NB = C::DP / 32, NBR = D / 32;
        uint8_t* qbuf = sQ + qb * 2 * C::Q_BYTES;
        uint8_t* sfbuf = sQsf + qb * 2 * C::SF_BYTES;
        const __half* qsl = args.q_in + static_cast<size_t>(item.slice) * args.seq_q * D;
        const int row_base = item.pair * 2 * C::BM;
        constexpr int kUnits = 2 * C::BM * NB;
        auto load = [&](int u, uint4 (&raw)[4]) {
            const int r = u / NB, b = u % NB, grow = row_base + r;
            const bool has = b < NBR && grow < args.seq_q;
            if (has) load_raw32(qsl + static_cast<size_t>(grow) * D + b * 32, raw);
            return has;
        };
        uint4 nxt[4];
        bool nxt_has = tid < kUnits && load(tid, nxt);
        for (int u = tid; u < kUnits; u += nthr) {
            uint4 cur[4];
#pragma unroll
            for (int k = 0; k < 4; k++) cur[k] = nxt[k];
            const bool has = nxt_has;
            nxt_has = u + nthr < kUnits && load(u + nthr, nxt);
            uint4 packed = make_uint4(0u, 0u, 0u, 0u);
            uint32_t sb = 127u;
            if (has) {
                float v[32];
                raw32_to_float(cur, v);
                sb = encode32<__half>(v, args.ocp_mode, packed);
                if (sb == 255u) sb = 254u;  // as the pre-pass stores it (255 is NaN in E8M0)
            }
            const int r = u / NB, b = u % NB, t = r / C::BM, rr = r % C::BM;
            // 16-byte unit b of a QK_ROW-byte row under the TMA's 64- or 32-byte swizzle.
            const int pu = C::QK_ROW == 64 ? (b ^ ((rr >> 1) & 3)) : (b ^ ((rr >> 2) & 1));
            *reinterpret_cast<uint4*>(qbuf + t * C::Q_BYTES + rr * C::QK_ROW + pu * 16) = packed;
            sfbuf[t * C::SF_BYTES + sf_tile_offset(128, rr, b)] = static_cast<uint8_t>(sb);
        }
        ptx::fence_proxy_async_smem();  // visible to the tensor cores' reads
    };

    if (warp < 4) {
        ptx::setmaxnreg_dec<PairRegs<kFuseQ>::kCtl>();
        if (warp == 0) {
            // -------------------------------------------------------- producer
            // Items in order; the K/V ring index kv runs on across items, and
            // the next item's Q (and its first K/V tiles) load while the
            // current item's last steps run.
            if (lane == 0) {
                int it = 0, kv = 0, k_issued = 0, v_issued = 0;
                bool ok = true;
                for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
                    const PairItem item = pair_item<kSmall>(args, r);
                    if (!item.valid) continue;
                    const int slice = item.slice, pair = item.pair, nk = item.nk;
                    uint64_t* qload = kFuseQ ? q_first : q_full;  // (kFuseQ: the first item only)
                    if (kFuseQ && it > 0) {
                        // Q of later items is quantised in the kernel (warp 3).
                    } else if (it > 0 && !wait_phase(q_empty, (it - 1) & 1, wctx, kSiteQEmpty)) {
                        break;
                    } else if constexpr (kSmall) {
                        const int qt = args.qtiles;
                        ptx::mbar_arrive_expect_tx(qload, qt * (C::Q_BYTES + C::SF_BYTES));
                        for (int t = 0; t < qt; t++) {
                            ptx::tma_load_3d(sQ + t * C::Q_BYTES, &tm_q, qload, 0, (pair * qt + t) * C::BM, slice);
                            ptx::bulk_load(sQsf + t * C::SF_BYTES,
                                           args.q_sf + (static_cast<size_t>(slice) * args.q_sf_tiles + qt * pair + t) *
                                                           C::SF_BYTES,
                                           C::SF_BYTES, qload);
                        }
                    } else {
                    ptx::mbar_arrive_expect_tx(qload, 2 * (C::Q_BYTES + C::SF_BYTES));
#pragma unroll
                    for (int t = 0; t < 2; t++) {
                        ptx::tma_load_3d(sQ + t * C::Q_BYTES, &tm_q, qload, 0, pair * 2 * C::BM + t * C::BM, slice);
                        ptx::bulk_load(sQsf + t * C::SF_BYTES,
                                       args.q_sf + (static_cast<size_t>(slice) * args.q_sf_tiles + 2 * pair + t) *
                                                       C::SF_BYTES,
                                       C::SF_BYTES, qload);
                    }
                    }
                    for (int jl = 0; jl < nk; jl++, kv++) {
                        const int j = kSmall ? item.k0 + jl : jl;  // key tile
                        const int ks = kv % C::KST;
                        if (kv >= C::KST && !wait_phase(&k_empty[ks], ((kv / C::KST) - 1) & 1, wctx, kSiteKEmpty)) {
                            ok = false;
                            break;
                        }
                        ptx::mbar_arrive_expect_tx(&k_full[ks], C::K_BYTES + C::SF_BYTES);
                        ptx::tma_load_3d(sK + ks * C::K_STRIDE, &tm_k, &k_full[ks], 0, j * BN, slice);
                        ptx::bulk_load(sKsf + ks * C::SF_BYTES,
                                       args.k_sf + (static_cast<size_t>(slice) * args.nk_tiles + j) * C::SF_BYTES, C::SF_BYTES,
                                       &k_full[ks]);
                        k_issued = kv + 1;
                        const int vs = kv % C::VST;
                        if (kv >= C::VST && !wait_phase(&v_empty[vs], ((kv / C::VST) - 1) & 1, wctx, kSiteVEmpty)) {
                            ok = false;
                            break;
                        }
                        ptx::mbar_arrive_expect_tx(&v_full[vs], C::V_BYTES);
#pragma unroll
                        for (int c = 0; c < C::VCH; c++)
                            ptx::tma_load_3d(sV + vs * C::V_STRIDE + c * BN * C::VCW, &tm_v, &v_full[vs],
                                             c * (C::VCW / 2), j * BN, slice);
                        v_issued = kv + 1;
                    }
                    it++;
                }
                // Every load this thread issued must land before the CTA exits
                // (Q loads are at most one phase ahead of their consumer).
                const unsigned long long drain_ns = 2ull * args.timeout_ns;
                if (it > 0) drain_phase(kFuseQ ? q_first : q_full, kFuseQ ? 0 : (it - 1) & 1, drain_ns);
                for (int i = k_issued - C::KST < 0 ? 0 : k_issued - C::KST; i < k_issued; i++)
                    drain_phase(&k_full[i % C::KST], (i / C::KST) & 1, drain_ns);
                for (int i = v_issued - C::VST < 0 ? 0 : v_issued - C::VST; i < v_issued; i++)
                    drain_phase(&v_full[i % C::VST], (i / C::VST) & 1, drain_ns);
            }
            __syncwarp();
        } else if (warp == 1) {
            // -------------------------------------------------------- S_t = Q_t K^T issuer
            if (lane == 0) {
                constexpr uint32_t qk_layout = ptx::swizzle_mode_for_bytes(C::CW);
                const uint64_t qdesc0 = ptx::make_sdesc(ptx::smem_u32(sQ), 16, 8 * C::CW, qk_layout);
                const uint64_t kdesc0 = ptx::make_sdesc(ptx::smem_u32(sK), 16, 8 * C::CW, qk_layout);
                const uint64_t sfdesc0 = ptx::make_sdesc(ptx::smem_u32(sQsf), 0, 128, ptx::kSwizzleNone);
                const uint64_t ksfdesc0 = ptx::make_sdesc(ptx::smem_u32(sKsf), 0, 128, ptx::kSwizzleNone);
                // g: global step (s_free phase), kv: K ring index, it: item.
                int g = 0, kv = 0, it = 0;
                bool ok = true;
                for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
                    const PairItem item = pair_item<kSmall>(args, r);
                    if (!item.valid) continue;
                    const int nk = item.nk;
                    // kFuseQ: item it reads Q buffer it & 1; item 0 comes by TMA
                    // (q_first), and item it > 0 is warp 3's ci-th item in that
                    // buffer (buffer 0 holds items 2, 4, ..., buffer 1 items 1, 3, ...).
                    const int qb = kFuseQ ? (it & 1) : 0;
                    const int ci = (it >> 1) - (qb == 0 ? 1 : 0);
                    uint64_t* qwait = !kFuseQ ? q_full : it == 0 ? q_first : qf(qb);
                    if (!wait_phase(qwait, !kFuseQ ? it & 1 : it == 0 ? 0 : ci & 1, wctx, kSiteQFull)) break;
                    ptx::tc_fence_after();
                    // The previous item's S MMAs are complete: the producer
                    // loaded this Q only after their q_empty commit arrived.
                    const uint32_t sfa = tmem + C::SFA_COL;
                    const int qt = kSmall ? args.qtiles : 2;
#pragma unroll
                    for (int t = 0; t < 2; t++)
                        if (t < qt)
                            ptx::tc_cp_32x128b_warpx4(sfa + 4 * t, sfdesc0 + static_cast<uint64_t>(((qb * 2 + t) * C::SF_BYTES) >> 4));
                    for (int j = 0; ok && j < nk; j++, kv++, g++) {
                        const int ks = kv % C::KST;
                        if (!wait_phase(&k_full[ks], (kv / C::KST) & 1, wctx, kSiteKFull)) { ok = false; break; }
                        ptx::tc_fence_after();
                        const uint32_t sfb = tmem + C::SFB_COL + 4 * ks;
                        ptx::tc_cp_32x128b_warpx4(sfb, ksfdesc0 + static_cast<uint64_t>((ks * C::SF_BYTES) >> 4));
                        const uint64_t kdesc = kdesc0 + static_cast<uint64_t>((ks * C::K_STRIDE) >> 4);
#pragma unroll
                        for (int t = 0; t < 2; t++) {
                            if (t >= qt) break;
                            // S_t's columns are free once warpgroup t holds the previous step in registers.
                            if (g > 0) {
                                if (!wait_phase(&s_free[t], (g - 1) & 1, wctx, kSiteSFree)) { ok = false; break; }
                                ptx::tc_fence_after();
                            }
#pragma unroll
                            for (int kk = 0; kk < C::KSTEPS; kk++) {
                                const uint32_t sf_id = 2u * (kk & 1);
                                ptx::mma_mxf4(tmem + C::S_COL + t * BN,
                                              qdesc0 + static_cast<uint64_t>(((qb * 2 + t) * C::Q_BYTES + kk * 32) >> 4),
                                              kdesc + static_cast<uint64_t>((kk * 32) >> 4),
                                              ptx::idesc_mxf4(128, BN, sf_id, sf_id), (sfa + 4 * t) | (sf_id << 30),
                                              sfb | (sf_id << 30), kk > 0 ? 1u : 0u);
                            }
                            ptx::tc_commit(&s_full[t]);
                        }
                        if (!ok) break;
                        ptx::tc_commit(&k_empty[ks]);
                    }
                    if (!ok) break;
                    ptx::tc_commit(kFuseQ ? qe(qb) : q_empty);  // the next Q may be written into this buffer
                    it++;
                }
                // Drain every tcgen05 op this thread issued before TMEM is freed.
                ptx::tc_commit(drain_bar);
                drain_phase(drain_bar, 0, 2ull * args.timeout_ns);
            }
            __syncwarp();
        } else if (warp == 2) {
            // -------------------------------------------------------- O_t += P_t V issuer
            if (lane == 0) {
                constexpr uint32_t v_layout = ptx::swizzle_mode_for_bytes(C::VCW);
                const uint64_t vdesc0 = ptx::make_sdesc(ptx::smem_u32(sV), BN * C::VCW, 8 * C::VCW, v_layout);
                constexpr uint32_t idesc_pv = ptx::idesc_f16(128, C::NPV, true);
                int g = 0;  // global step: p_full phase and V ring index
                bool ok = true;
                for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
                    const PairItem item = pair_item<kSmall>(args, r);
                    if (!item.valid) continue;
                    const int nk = item.nk;
                    for (int j = 0; ok && j < nk; j++, g++) {
                        const int vs = g % C::VST;
                        if (!wait_phase(&v_full[vs], (g / C::VST) & 1, wctx, kSiteVFull)) { ok = false; break; }
                        const uint64_t vdesc = vdesc0 + static_cast<uint64_t>((vs * C::V_STRIDE) >> 4);
#pragma unroll
                        for (int t = 0; t < 2; t++) {
                            if (kSmall && t >= args.qtiles) break;
                            if (!wait_phase(&p_full[t], g & 1, wctx, kSitePFull)) { ok = false; break; }
                            ptx::tc_fence_after();
                            // The first step of an item starts O_t afresh.
#pragma unroll
                            for (int kk = 0; kk < BN / 16; kk++)
                                ptx::mma_f16_ts(tmem + C::O_COL + t * C::NPV, tmem + C::P_COL + t * (BN / 2) + kk * 8,
                                                vdesc + static_cast<uint64_t>((kk * 16 * C::VCW) >> 4), idesc_pv,
                                                (j > 0 || kk > 0) ? 1u : 0u);
                            ptx::tc_commit(&pv_done[t]);
                        }
                        if (!ok) break;
                        ptx::tc_commit(&v_empty[vs]);
                    }
                }
                ptx::tc_commit(drain_bar);
                drain_phase(drain_bar, 0, 2ull * args.timeout_ns);
            }
            __syncwarp();
        } else if constexpr (kFuseQ) {
            // -------------------------------------------------------- warp 3: Q quantiser
            // Items after the CTA's first, each into the Q buffer its S MMAs
            // will read, once the item two back is done with that buffer.
            int it = 0;
            for (int r = 0; r * static_cast<int>(gridDim.x) < args.n_items; r++) {
                const PairItem item = pair_item<kSmall>(args, r);
                if (!item.valid) continue;
                if (it > 0) {
                    const int qb = it & 1;
                    if (it >= 2 && !__all_sync(0xffffffffu, wait_phase(qe(qb), ((it >> 1) - 1) & 1, wctx, kSiteQEmpty)))
                        break;
                    quantize_q(item, qb, lane, 32);
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(qf(qb));
                }
                it++;
            }
        }
    } else {
        ptx::setmaxnreg_inc<PairRegs<kFuseQ>::kSm>();
        // ------------------------------------------------------------ softmax warpgroups
        constexpr int NT = BN / 32;                // 32-column chunks of an S row
        const int t = (warp - 4) / 4;              // query tile of this warpgroup
        const int wq = warp & 3;                   // TMEM lane quarter this warp may access
        const int row = wq * 32 + lane;            // query row within the tile
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t s_tm = tmem + lane_off + C::S_COL + t * BN;
        const uint32_t o_tm = tmem + lane_off + C::O_COL + t * C::NPV;
        const uint32_t p_tm = tmem + lane_off + C::P_COL + t * (BN / 2);
        const float c = args.scale_log2;
        uint8_t* ost = smem + C::OFF_OST + (warp - 4) * 2 * C::OST_BYTES;
        // kSmall: the end of an item of tile t, once its last P.V is done.
        // Without key partitions O / l goes to the output; with them the item
        // stores its partials and, if it completes its group, merges them.
        // Returns false when a wait gave up.
        auto small_epilogue = [&](const PairItem& item, float m_ref, int& splits) -> bool {
            ptx::tc_fence_after();
            uint32_t lsum[16];
            ptx::tmem_ld16(o_tm + C::L_COL, lsum);
            ptx::tc_wait_ld();
            const float lv = __uint_as_float(lsum[0]);
            const int trow0 = (item.pair * args.qtiles + t) * C::BM;  // first query row of this tile
            // 32-column chunks of this warp's 32 rows: staged swizzled like the
            // TMA box (so a warp's 16-byte writes hit distinct banks), then one
            // lane stores the box with TMA (rows past the map's end are
            // clipped).  src(k, o) fills o with chunk k of this thread's row.
            auto store_rows = [&](auto src, auto as_f32, const CUtensorMap* map, int row0, int slice_coord,
                                  float scale) {
                constexpr bool f32 = decltype(as_f32)::value || sizeof(OutT) == 4;
                constexpr int OB = f32 ? 128 : 64;  // bytes per staged row
                if (lane == 0) ptx::bulk_wait_group_read<0>();
                __syncwarp();
#pragma unroll 1
                for (int k = 0; k < D / 32; k++) {
                    uint32_t o[32];
                    src(k, o);
                    uint8_t* buf = ost + (k & 1) * C::OST_BYTES;
                    if (k >= 2) {
                        if (lane == 0) ptx::bulk_wait_group_read<1>();
                        __syncwarp();
                    }
                    uint32_t ov[OB / 4];
                    if constexpr (f32) {
#pragma unroll
                        for (int i = 0; i < 32; i++) ov[i] = __float_as_uint(__uint_as_float(o[i]) * scale);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            ov[i] = ptx::pack_half2(__uint_as_float(o[2 * i]) * scale, __uint_as_float(o[2 * i + 1]) * scale);
                    }
#pragma unroll
                    for (int u = 0; u < OB / 16; u++) {
                        const int pu = OB == 128 ? (u ^ (lane & 7)) : (u ^ ((lane >> 1) & 3));
                        *reinterpret_cast<uint4*>(buf + lane * OB + pu * 16) =
                            make_uint4(ov[4 * u], ov[4 * u + 1], ov[4 * u + 2], ov[4 * u + 3]);
                    }
                    ptx::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        ptx::tma_store_3d(map, buf, 32 * k, row0, slice_coord);
                        ptx::bulk_commit_group();
                    }
                }
            };
            auto from_tmem = [&](int k, uint32_t (&o)[32]) {
                ptx::tmem_ld32(o_tm + 32 * k, o);
                ptx::tc_wait_ld();
            };
            if (args.kparts == 1) {
                const float inv_l = lv > 0.f ? 1.0f / lv : 0.f;  // a row that saw no key outputs 0
                if constexpr (kLse) {
                    if (trow0 + row < args.seq_q)
                        args.lse[static_cast<size_t>(item.slice) * args.seq_q + trow0 + row] =
                            lv > 0.f ? (m_ref + log2f(lv)) * kLn2 : INFINITY;
                }
                store_rows(from_tmem, std::false_type{}, &tm_o, trow0 + wq * 32, item.slice, inv_l);
                return true;
            }
            // ---- a key partition: its partials ----
            const int prow0 = (item.idx * args.qtiles + t) * C::BM;  // this tile's rows in the partials
            args.part_ml[prow0 + row] = make_float2(m_ref, lv);
            store_rows(from_tmem, std::true_type{}, &tm_p, prow0 + wq * 32, 0, 1.0f);
            // Visible to the CTA that merges the group: every lane's (m, l), then
            // lane 0's TMA stores once they are complete.
            __threadfence();
            __syncwarp();
            if (lane == 0) {
                ptx::bulk_wait_group<0>();
                ptx::fence_proxy_async_global();
                __threadfence();
                ptx::mbar_arrive(part_done);
            }
            if (warp == 4) {
                // Every softmax warp of this CTA has written its partials: count
                // this partition; the CTA that brings the count to kparts merges
                // (and leaves the counter at zero for the next launch).
                const bool all_in = __all_sync(0xffffffffu, wait_phase(part_done, splits & 1, wctx, kSitePartDone));
                int last = 0;
                if (all_in && lane == 0) {
                    __threadfence();
                    const unsigned prev = atomicAdd(&args.part_count[item.idx / args.kparts], 1u);
                    last = prev + 1 == static_cast<unsigned>(args.kparts);
                    if (last) {
                        atomicExch(&args.part_count[item.idx / args.kparts], 0u);
                        __threadfence();
                    }
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (lane == 0) {
                    merge_sh = last;
                    ptx::mbar_arrive(merge_go);
                }
            }
            if (!__all_sync(0xffffffffu, wait_phase(merge_go, splits & 1, wctx, kSitePartDone))) return false;
            splits++;
            if (!merge_sh) return true;
            // ---- the group's last partition: merge the kparts partitions ----
            // O = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p, M = max_p m_p.
            // Lane i first forms the weights w_p = 2^(m_p - M) / L of row i of
            // this warp; then the warp walks its 32 rows in batches, each row
            // read whole by the 32 lanes (D/32 columns each: coalesced), the
            // batch's rows x 4 partitions of loads issued together, and
            // writes the output rows directly (rows past seq_q are skipped).
            const int gbase = (item.idx / args.kparts) * args.kparts;
            auto prow = [&](int pp, int rr) { return ((gbase + pp) * args.qtiles + t) * C::BM + wq * 32 + rr; };
            float wgt[kMaxKParts];
            {
                float mp[kMaxKParts], lp[kMaxKParts];
#pragma unroll
                for (int pp = 0; pp < kMaxKParts; pp++) {
                    const float2 ml = __ldcg(&args.part_ml[prow(pp < args.kparts ? pp : 0, lane)]);
                    mp[pp] = pp < args.kparts ? ml.x : -INFINITY;
                    lp[pp] = ml.y;
                }
                float row_m = -INFINITY;
#pragma unroll
                for (int pp = 0; pp < kMaxKParts; pp++) row_m = fmaxf(row_m, mp[pp]);
                float lsum_all = 0.f;
#pragma unroll
                for (int pp = 0; pp < kMaxKParts; pp++) {
                    wgt[pp] = mp[pp] == -INFINITY ? 0.f : ptx::ex2_approx(mp[pp] - row_m);
                    lsum_all = fmaf(wgt[pp], lp[pp], lsum_all);
                }
                const float row_inv = lsum_all > 0.f ? 1.0f / lsum_all : 0.f;  // a row that saw no key outputs 0
#pragma unroll
                for (int pp = 0; pp < kMaxKParts; pp++) wgt[pp] *= row_inv;
                if constexpr (kLse) {
                    if (trow0 + wq * 32 + lane < args.seq_q)
                        args.lse[static_cast<size_t>(item.slice) * args.seq_q + trow0 + wq * 32 + lane] =
                            lsum_all > 0.f ? (row_m + log2f(lsum_all)) * kLn2 : INFINITY;
                }
            }
            constexpr int CPL = D / 32;            // output columns per lane
            constexpr int RB = CPL >= 3 ? 4 : 8;   // rows per batch
            const int rows_here = min(32, args.seq_q - (trow0 + wq * 32));
#pragma unroll 1
            for (int r0 = 0; r0 < rows_here; r0 += RB) {
                float acc[RB][CPL];
#pragma unroll
                for (int u = 0; u < RB; u++)
#pragma unroll
                    for (int c = 0; c < CPL; c++) acc[u][c] = 0.f;
#pragma unroll
                for (int pg = 0; pg < kMaxKParts; pg += 4) {
                    if (pg >= args.kparts) break;
                    float v[4][RB][CPL];
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        // A partition past kparts reads partition pg again (weight 0).
                        const int pp = pg + q < args.kparts ? pg + q : pg;
#pragma unroll
                        for (int u = 0; u < RB; u++) {
                            const float* src = args.part_o + static_cast<size_t>(prow(pp, r0 + u)) * D + lane * CPL;
                            if constexpr (CPL == 4) {
                                const float4 x = __ldcg(reinterpret_cast<const float4*>(src));
                                v[q][u][0] = x.x; v[q][u][1] = x.y; v[q][u][2] = x.z; v[q][u][3] = x.w;
                            } else if constexpr (CPL == 2) {
                                const float2 x = __ldcg(reinterpret_cast<const float2*>(src));
                                v[q][u][0] = x.x; v[q][u][1] = x.y;
                            } else {
#pragma unroll
                                for (int c = 0; c < CPL; c++) v[q][u][c] = __ldcg(src + c);
                            }
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 4; q++)
#pragma unroll
                        for (int u = 0; u < RB; u++) {
                            const float w = __shfl_sync(0xffffffffu, wgt[pg + q], (r0 + u) & 31);
#pragma unroll
                            for (int c = 0; c < CPL; c++) acc[u][c] = fmaf(w, v[q][u][c], acc[u][c]);
                        }
                }
#pragma unroll
                for (int u = 0; u < RB; u++) {
                    if (r0 + u >= rows_here) break;
                    const size_t orow = static_cast<size_t>(item.slice) * args.seq_q + trow0 + wq * 32 + r0 + u;
                    OutT* dst = static_cast<OutT*>(args.out) + orow * D + lane * CPL;
#pragma unroll
                    for (int c = 0; c < CPL; c++) {
                        if constexpr (sizeof(OutT) == 4) dst[c] = acc[u][c];
                        else dst[c] = __float2half_rn(acc[u][c]);
                    }
                }
            }
            return true;
        };
        int g = 0;  // global step: phase of s_full / s_free / p_full / pv_done
        int splits = 0;  // kSmall: items of split groups so far (phase of part_done / merge_go)
        bool ok = !kSmall || t < args.qtiles;  // with one query tile per item, warpgroup 1 has no work
        for (int r = 0; ok && r * static_cast<int>(gridDim.x) < args.n_items; r++) {
            const PairItem item = pair_item<kSmall>(args, r);
            if (!item.valid) continue;
            const int slice = item.slice, pair = item.pair, nk = item.nk;
            // Keys this row sees: [0, row_lim) (the causal mask, or all keys).
            const int qi = kSmall ? (pair * args.qtiles + t) * C::BM + row : pair * 2 * C::BM + t * C::BM + row;
            const int row_lim = args.causal ? min(qi + args.causal_off + 1, args.seq_k) : args.seq_k;
            float m = -INFINITY;
            for (int j = 0; j < nk; j++, g++) {
                if (!__all_sync(0xffffffffu, wait_phase(&s_full[t], g & 1, wctx, kSiteSFull))) { ok = false; break; }
                ptx::tc_fence_after();
                uint32_t sr[NT][32];
#pragma unroll
                for (int k = 0; k < NT; k++) ptx::tmem_ld32(s_tm + 32 * k, sr[k]);
                ptx::tc_wait_ld();
                // S_t is in registers: the issuer may compute the next step into it.
                ptx::tc_fence_before();
                if (!kWithhold || threadIdx.x != 128 || g != 0) ptx::mbar_arrive(&s_free[t]);
                const int valid = row_lim - (kSmall ? item.k0 + j : j) * BN;  // keys of this step this row sees
                uint32_t pk[NT][16];
                // P = 2^(S * c - mref) as FP16 pairs; kPoly8 of every 8 column
                // pairs take 2^x on the FMA pipe, the rest on MUFU.  With a true
                // tag it also returns the row max of S, whose (independent) ALU
                // work then interleaves with the exponentials.
                auto exps = [&](float mref, auto with_max) -> float {
                    const float2 c2 = make_float2(c, c), nm2 = make_float2(-mref, -mref);
                    float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                    for (int k = 0; k < NT; k++)
#pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            const float s0 = __uint_as_float(sr[k][i]), s1 = __uint_as_float(sr[k][i + 1]);
                            if constexpr (decltype(with_max)::value) mx4[(i >> 1) & 3] = ptx::fmax3(mx4[(i >> 1) & 3], s0, s1);
                            const float2 x = ptx::ffma2(make_float2(s0, s1), c2, nm2);
                            const float2 p = ((i >> 1) & 7) < kPoly8 ? ptx::exp2_poly3(x)
                                                                     : make_float2(ptx::ex2_approx(x.x), ptx::ex2_approx(x.y));
                            pk[k][i / 2] = ptx::pack_half2(p.x, p.y);
                        }
                    return ptx::fmax3(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3]));
                };
                float alpha = 1.f;
                bool rescale = false;
                bool exact = true;
                float spec_mx = 0.f;  // row max from the speculative pass, when it ran
                const bool spec_ok =
                    args.causal ? __all_sync(0xffffffffu, valid >= BN && m != -INFINITY) : valid >= BN;
                if (kSpec && j > 0 && spec_ok) {
                    // Speculative pass against the current reference max m: it
                    // stands unless some row's max grew by more than 2^15 (the lazy
                    // rescale threshold), which after the first step is rare.
                    const float mx = exps(m, std::true_type{});
                    spec_mx = mx;
                    exact = __any_sync(0xffffffffu, mx * c > m + kLazyRescaleLog2);
                }
                if (exact && __all_sync(0xffffffffu, valid <= 0)) {
                    // No row of this warp sees a key of this step: P = 0.
#pragma unroll
                    for (int k = 0; k < NT; k++)
#pragma unroll
                        for (int i = 0; i < 16; i++) pk[k][i] = 0u;
                } else if (exact) {
                    // Row max first, then the exponentials: the first step, the
                    // ragged or masked steps, and steps where some row's max jumped.
                    float row_max;
                    if (kSpec && j > 0 && spec_ok) {
                        row_max = spec_mx;  // a failed speculative pass already formed it (no masking there)
                    } else {
                        if (valid < BN) {
#pragma unroll
                            for (int k = 0; k < NT; k++)
#pragma unroll
                                for (int i = 0; i < 32; i++)
                                    if (32 * k + i >= valid) sr[k][i] = __float_as_uint(-INFINITY);
                        }
                        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                        for (int k = 0; k < NT; k++)
#pragma unroll
                            for (int i = 0; i < 32; i += 2)
                                mx4[(i >> 1) & 3] = ptx::fmax3(mx4[(i >> 1) & 3], __uint_as_float(sr[k][i]),
                                                               __uint_as_float(sr[k][i + 1]));
                        row_max = ptx::fmax3(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3]));
                    }
                    const float m_new = fmaxf(m, row_max * c);
                    if (j == 0) {
                        m = m_new;
                    } else if (m_new > m + kLazyRescaleLog2) {
                        // Lazy rescale: O and l keep the old reference max until
                        // the row max has grown by more than 2^15.
                        alpha = ptx::ex2_approx(m - m_new);
                        m = m_new;
                        rescale = true;
                    }
                    // A row that has seen no key yet keeps m = -inf; its P is 0.
                    (void)exps(m == -INFINITY ? 0.f : m, std::false_type{});
                }
                if (j > 0) {
                    // PV_{j-1} must be done: it reads the P columns this step
                    // overwrites, and O is rescaled below.
                    if (!__all_sync(0xffffffffu, wait_phase(&pv_done[t], (g - 1) & 1, wctx, kSitePvDone))) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                }
#pragma unroll
                for (int k = 0; k < NT; k++) ptx::tmem_st16(p_tm + 16 * k, pk[k]);
                if (j > 0 && __any_sync(0xffffffffu, rescale)) {
                    // O and its row-sum columns move to the new reference max.
#pragma unroll 1
                    for (int k = 0; k < C::L_COL / 32; k++) {
                        uint32_t o[32];
                        ptx::tmem_ld32(o_tm + 32 * k, o);
                        ptx::tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        ptx::tmem_st32(o_tm + 32 * k, o);
                    }
                    uint32_t o[16];
                    ptx::tmem_ld16(o_tm + C::L_COL, o);
                    ptx::tc_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    ptx::tmem_st16(o_tm + C::L_COL, o);
                }
                ptx::tc_wait_st();
                ptx::tc_fence_before();
                ptx::mbar_arrive(&p_full[t]);
            }
            // The last step's P.V must be complete before O is read.
            if (!ok || !__all_sync(0xffffffffu, wait_phase(&pv_done[t], (g - 1) & 1, wctx, kSitePvDone))) {
                ok = false;
                break;
            }
            if constexpr (kSmall) {
                if (!small_epilogue(item, m, splits)) {
                    ok = false;
                    break;
                }
            } else
            {
                ptx::tc_fence_after();
                uint32_t lsum[16];
                ptx::tmem_ld16(o_tm + C::L_COL, lsum);
                ptx::tc_wait_ld();
                const float lv = __uint_as_float(lsum[0]);
                const float inv_l = lv > 0.f ? 1.0f / lv : 0.f;  // a row that saw no key outputs 0
                if constexpr (kLse) {
                    const int grow = pair * 2 * C::BM + t * C::BM + row;
                    if (grow < args.seq_q)
                        args.lse[static_cast<size_t>(slice) * args.seq_q + grow] =
                            lv > 0.f ? (m + log2f(lv)) * kLn2 : INFINITY;
                }
                // O / l in 32-column chunks: each warp writes its 32 rows x 32
                // columns to a staging buffer (swizzled like the TMA box, so the
                // 16-byte writes of a warp hit distinct banks) and lane 0 stores
                // the box with TMA; rows past seq_q are clipped by the tensor map.
                constexpr int OB = 32 * static_cast<int>(sizeof(OutT));  // bytes per staged row
                const int grow0 = pair * 2 * C::BM + t * C::BM + wq * 32;
                // The previous item's stores (long finished) must be done
                // reading the staging buffers before they are rewritten.
                if (lane == 0) ptx::bulk_wait_group_read<0>();
                __syncwarp();
                // The warp's staging (2 x OST_BYTES) holds NSLOT chunks: they
                // are written, then made visible to the TMA with one proxy
                // fence, and stored as a group.
                constexpr int CB = 32 * OB;
                constexpr int NSLOT = 2 * C::OST_BYTES / CB;
#pragma unroll 1
                for (int k = 0; k < D / 32; k++) {
                    uint32_t o[32];
                    ptx::tmem_ld32(o_tm + 32 * k, o);
                    ptx::tc_wait_ld();
                    const int slot = k % NSLOT;
                    uint8_t* buf = ost + slot * CB;
                    if (k >= NSLOT && slot == 0) {
                        // The previous group's stores must be done reading the staging.
                        if (lane == 0) ptx::bulk_wait_group_read<0>();
                        __syncwarp();
                    }
                    uint32_t ov[OB / 4];
                    if constexpr (sizeof(OutT) == 4) {
#pragma unroll
                        for (int i = 0; i < 32; i++) ov[i] = __float_as_uint(__uint_as_float(o[i]) * inv_l);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            ov[i] = ptx::pack_half2(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
                    }
#pragma unroll
                    for (int u = 0; u < OB / 16; u++) {
                        const int pu = OB == 128 ? (u ^ (lane & 7)) : (u ^ ((lane >> 1) & 3));
                        *reinterpret_cast<uint4*>(buf + lane * OB + pu * 16) =
                            make_uint4(ov[4 * u], ov[4 * u + 1], ov[4 * u + 2], ov[4 * u + 3]);
                    }
                    if (slot == NSLOT - 1 || k == D / 32 - 1) {
                        ptx::fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            for (int kk = k - slot; kk <= k; kk++)
                                ptx::tma_store_3d(&tm_o, ost + (kk % NSLOT) * CB, 32 * kk, grow0, slice);
                            ptx::bulk_commit_group();
                        }
                    }
                }
            }
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

}  // namespace fp4attn
