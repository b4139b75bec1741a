// fp4attn.cu -- the C ABI of libfp4attn.so (declared in include/fp4attn.h):
// argument checking, workspace layout, TMA tensor maps and kernel dispatch.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/fp4attn.h"
#include "attention_pair.cuh"
#include "quantize.cuh"

namespace fp4attn {

// Unique id of the calling thread's current CUDA context (cuCtxGetId; an id
// is never reused within a process), or 0 when no context is current yet or
// the driver lacks the call.  Per-device state that a device reset would
// invalidate (kernel attributes, symbol addresses) is keyed on it.
unsigned long long current_context_id()
{
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    });
    if (!get_current || !get_id) return 0;
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
    unsigned long long id = 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

}  // namespace fp4attn

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define FP4_CUDA(call)                                                                              \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) return fail(FP4ATTN_ECUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

constexpr int kSupportedDims[] = {32, 64, 96, 128, 160, 256};

bool supported_dim(int d)
{
    for (int x : kSupportedDims)
        if (x == d) return true;
    return false;
}

// Keys per attention step: 64 (the two-query-tile kernel for head_dim <= 128,
// and head_dim 256), except head_dim 160 (one query tile, 128 keys).
int block_n_for(int d) { return d == 160 ? 128 : 64; }
// The two-query-tile kernel covers head_dim <= 128.
bool paired(int d) { return d <= 128; }
int padded_dim(int d) { return (d + 63) / 64 * 64; }
int sfa_atoms(int d) { return (padded_dim(d) + 127) / 128; }
int sf_tile_bytes(int d, int tile_rows)
{
    return tile_rows == 128 ? 512 * sfa_atoms(d) : 512 * ((padded_dim(d) + 255) / 256);
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct Workspace {
    size_t q_codes, k_codes, q_sf, k_sf, v16, part_o, part_ml, part_count, total;
};

// 128-row Q scale tiles per slice: rounded up to whole pairs for the
// two-query-tile kernel (the extra tile holds padding scales).
int q_sf_tiles(int sq, int d)
{
    const int nq = (sq + 127) / 128;
    return paired(d) ? (nq + 1) / 2 * 2 : nq;
}

// Key partitions per query group are capped by this many work items in all:
// about one per SM of a B200 (148).  A fixed number, so that the workspace
// size is a function of the shape alone.
constexpr int kSplitItems = 148;

// Fewest 64-key tiles a key partition gets (below that the partial results
// and their merge cost more than the shorter key loop saves).
// FP4ATTN_KSPLIT overrides it for tuning; 0 keeps every query group on one CTA.
int ksplit_min_tiles()
{
    static int v = [] {
        const char* s = getenv("FP4ATTN_KSPLIT");
        return s ? atoi(s) : 4;
    }();
    return v;
}

// Schedule of the two-query-tile kernel for a problem: one query tile per
// item when seq_q <= 128, otherwise pairs; and, when there are fewer query
// groups than kSplitItems (and no mask), the keys of each group split into
// kparts partitions of nk_part 64-key tiles, each its own work item.
struct PairPlan {
    int qtiles, n_pairs, kparts, nk_part;
    int64_t groups;
};

PairPlan pair_plan(int64_t slices, int sq, int sk, int d, bool causal)
{
    PairPlan p;
    const int nq = (sq + 127) / 128;
    p.qtiles = nq == 1 ? 1 : 2;
    p.n_pairs = p.qtiles == 1 ? 1 : q_sf_tiles(sq, d) / 2;
    p.groups = slices * p.n_pairs;
    const int nk = (sk + 63) / 64;
    p.kparts = 1;
    p.nk_part = nk;
    const int min_tiles = ksplit_min_tiles();
    if (!causal && min_tiles > 0 && nk >= 2 * min_tiles && p.groups * 2 <= kSplitItems) {
        const int want = static_cast<int>(
            std::min<int64_t>(std::min<int64_t>(nk / min_tiles, kSplitItems / p.groups), fp4attn::kMaxKParts));
        p.nk_part = (nk + want - 1) / want;
        p.kparts = (nk + p.nk_part - 1) / p.nk_part;
    }
    return p;
}

Workspace plan_workspace(int64_t slices, int sq, int sk, int d, int in_dtype)
{
    const int dp = padded_dim(d), bn = block_n_for(d);
    const int64_t nq = q_sf_tiles(sq, d), nk = (sk + bn - 1) / bn;
    Workspace w{};
    size_t off = 0;
    w.q_codes = off;
    off = align256(off + static_cast<size_t>(slices) * sq * (dp / 2));
    w.k_codes = off;
    off = align256(off + static_cast<size_t>(slices) * sk * (dp / 2));
    w.q_sf = off;
    off = align256(off + static_cast<size_t>(slices) * nq * sf_tile_bytes(d, 128));
    w.k_sf = off;
    off = align256(off + static_cast<size_t>(slices) * nk * sf_tile_bytes(d, bn));
    w.v16 = off;
    if (in_dtype == FP4ATTN_F32) off = align256(off + static_cast<size_t>(slices) * sk * d * 2);
    // Key-partition partials of the two-query-tile kernel (see pair_plan).
    w.part_o = w.part_ml = w.part_count = off;
    if (paired(d)) {
        const PairPlan pp = pair_plan(slices, sq, sk, d, false);
        if (pp.kparts > 1) {
            const size_t rows = static_cast<size_t>(pp.groups) * pp.kparts * pp.qtiles * 128;
            w.part_o = off;
            off = align256(off + rows * d * 4);
            w.part_ml = off;
            off = align256(off + rows * 8);
            w.part_count = off;
            off = align256(off + static_cast<size_t>(pp.groups) * 4);
        }
    }
    w.total = off;
    return w;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Recently encoded tensor maps of this host thread.  A map is a pure function
// of its arguments (no device state), so a repeated call with the same
// pointers and shape -- a serving loop, a benchmark -- reuses the encoding.
struct MapKey {
    const void* base;
    uint64_t inner, rows, slices;
    uint32_t box_inner, box_rows;
    int dt, sw;
    bool operator==(const MapKey& o) const
    {
        return base == o.base && inner == o.inner && rows == o.rows && slices == o.slices &&
               box_inner == o.box_inner && box_rows == o.box_rows && dt == o.dt && sw == o.sw;
    }
};
struct MapCache {
    static constexpr int kEntries = 16;
    MapKey key[kEntries];
    CUtensorMap map[kEntries];
    int used = 0, next = 0;
};
thread_local MapCache g_map_cache;

// 3-D tensor map over [slices][rows][inner] with a (box_inner, box_rows, 1)
// box; rows past `rows` read as zero.
int make_map_3d(CUtensorMap* m, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t inner,
                uint64_t rows, uint64_t slices, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw)
{
    const MapKey key{base, inner, rows, slices, box_inner, box_rows, static_cast<int>(dt), static_cast<int>(sw)};
    MapCache& c = g_map_cache;
    for (int i = 0; i < c.used; i++)
        if (c.key[i] == key) {
            *m = c.map[i];
            return FP4ATTN_OK;
        }
    auto enc = tensor_map_encoder();
    if (!enc) return fail(FP4ATTN_ECUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {inner, rows, slices};
    cuuint64_t strides[2] = {inner * elem_bytes, inner * rows * elem_bytes};
    cuuint32_t box[3] = {box_inner, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FP4ATTN_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    const int slot = c.used < MapCache::kEntries ? c.used++ : c.next;
    c.next = (slot + 1) % MapCache::kEntries;
    c.key[slot] = key;
    c.map[slot] = *m;
    return FP4ATTN_OK;
}

CUtensorMapSwizzle swizzle_for(int bytes)
{
    return bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
}

// Per-device set-up, done once per device on its first use from any host
// thread: check for an sm_100 GPU and record its SM count.  Nothing is
// uploaded: the scale-rule table is initialised in the module image.
constexpr int kMaxDevices = 64;
struct DeviceState {
    bool done = false;
    int status = FP4ATTN_OK;
    std::string msg;
    int sms = 0;
};
std::mutex g_dev_mu;
DeviceState g_dev[kMaxDevices];

int current_device(int* dev)
{
    if (cudaGetDevice(dev) != cudaSuccess) return fail(FP4ATTN_ECUDA, "no CUDA device");
    if (*dev < 0 || *dev >= kMaxDevices) return fail(FP4ATTN_EUNSUPPORTED, "device index %d", *dev);
    return FP4ATTN_OK;
}

int device_ready()
{
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_dev_mu);
    DeviceState& d = g_dev[dev];
    if (!d.done) {
        d.done = true;
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
            d.status = FP4ATTN_ECUDA;
            d.msg = "could not query the CUDA device";
        } else if (prop.major != 10 || prop.minor != 0) {
            // The library carries sm_100a code only; architecture-specific
            // code runs on exactly that compute capability.
            d.status = FP4ATTN_EUNSUPPORTED;
            d.msg = "libfp4attn requires an sm_100 (B200-class) GPU; found sm_" + std::to_string(prop.major) +
                    std::to_string(prop.minor);
        } else {
            d.sms = prop.multiProcessorCount;
        }
    }
    if (d.status != FP4ATTN_OK) return fail(d.status, "%s", d.msg.c_str());
    return FP4ATTN_OK;
}

// SM count of the current device (device_ready() has run on it).
int device_sms()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 1;
    std::lock_guard<std::mutex> lock(g_dev_mu);
    return g_dev[dev].sms > 0 ? g_dev[dev].sms : 1;
}

// Sets a kernel's dynamic shared memory limit once per device context;
// `done_ctx` (the context id it was last set in, per device) belongs to the
// calling launcher, i.e. to one kernel.  A device reset makes a new context,
// and the attribute is set again there.
template <typename Kern>
int set_smem_once(Kern kern, int bytes, std::atomic<unsigned long long> (&done_ctx)[kMaxDevices])
{
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    const unsigned long long ctx = fp4attn::current_context_id();
    if (ctx != 0 && done_ctx[dev].load(std::memory_order_acquire) == ctx) return FP4ATTN_OK;
    FP4_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done_ctx[dev].store(ctx, std::memory_order_release);
    return FP4ATTN_OK;
}

// FP4ATTN_PDL=0 launches the attention kernels without programmatic stream
// serialization (for comparison).
bool pdl_enabled()
{
    static bool v = [] {
        const char* s = getenv("FP4ATTN_PDL");
        return !(s && atoi(s) == 0);
    }();
    return v;
}

// Launches an attention kernel as the programmatic dependent of whatever
// precedes it in the stream (normally the quantiser): its launch and
// prologue overlap that grid's tail, and the kernel waits for that grid's
// completion (griddepcontrol.wait) before it reads the workspace.
template <typename... KArgs, typename... Args>
int launch_dependent(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                     Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    FP4_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
    return FP4ATTN_OK;
}

unsigned long long wait_timeout_ns()
{
    static unsigned long long ns = [] {
        const char* s = getenv("FP4ATTN_WAIT_TIMEOUT_MS");
        long ms = s ? atol(s) : 2000;
        if (ms < 1) ms = 1;
        return static_cast<unsigned long long>(ms) * 1000000ull;
    }();
    return ns;
}

int grid_for(int64_t work, int per_block = 256)
{
    int64_t b = (work + per_block - 1) / per_block;
    if (b > 148 * 32) b = 148 * 32;
    return static_cast<int>(b < 1 ? 1 : b);
}

fp4attn::QuantTileArgs quant_args(int64_t slices, int seq, int d, int tile_rows, int ntiles, int ocp)
{
    fp4attn::QuantTileArgs a;
    a.slices = slices;
    a.seq = seq;
    a.head_dim = d;
    a.padded_dim = padded_dim(d);
    a.tile_rows = tile_rows;
    a.tile_shift = tile_rows == 128 ? 7 : 6;
    a.ntiles = ntiles;
    a.sf_tile_bytes = sf_tile_bytes(d, tile_rows);
    a.ocp_mode = ocp;
    return a;
}

// Q and K quantised by one launch (grid z = 0 for Q, 1 for K), and with a V
// job (FP32 input) V converted to FP16 by the same launch (z = 2).
template <typename InT>
int launch_quant_qk(const fp4attn::QuantJob& q, const fp4attn::QuantJob& k, const fp4attn::VConvJob* v,
                    int64_t slices, cudaStream_t st)
{
    auto gx_for = [&](const fp4attn::QuantTileArgs& a) {
        const int per_slice = a.ntiles * a.tile_rows * (a.padded_dim / 32);
        return static_cast<int>(std::min<int64_t>((per_slice + 255) / 256, std::max<int64_t>(1, 148 * 32 / slices + 1)));
    };
    const fp4attn::VConvJob vj = *v;
    dim3 grid(std::max(gx_for(q.a), gx_for(k.a)), static_cast<unsigned>(slices), v->src ? 3 : 2);
    switch (q.a.padded_dim / 32) {
        case 2: fp4attn::quantize_tiles_kernel<InT, 2><<<grid, 256, 0, st>>>(q, k, vj); break;
        case 4: fp4attn::quantize_tiles_kernel<InT, 4><<<grid, 256, 0, st>>>(q, k, vj); break;
        case 6: fp4attn::quantize_tiles_kernel<InT, 6><<<grid, 256, 0, st>>>(q, k, vj); break;
        case 8: fp4attn::quantize_tiles_kernel<InT, 8><<<grid, 256, 0, st>>>(q, k, vj); break;
        default: return fail(FP4ATTN_EUNSUPPORTED, "padded head_dim %d", q.a.padded_dim);
    }
    FP4_CUDA(cudaGetLastError());
    return FP4ATTN_OK;
}

template <int D, int BN, typename OutT, bool kScores, int kPoly8>
int launch_fwd_poly(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const fp4attn::FwdArgs& a,
                    int64_t slices, cudaStream_t st)
{
    using C = fp4attn::FwdCfg<D, BN>;
    auto kern = fp4attn::fp4_attention_fwd_kernel<D, BN, OutT, kScores, kPoly8>;
    // The kernel re-splits its launch registers with setmaxnreg; refuse to
    // launch unless the pool it was given covers the split.
    static std::atomic<int> launch_regs_cache{-1};
    int launch_regs = launch_regs_cache.load(std::memory_order_relaxed);
    if (launch_regs < 0) {
        cudaFuncAttributes attr;
        FP4_CUDA(cudaFuncGetAttributes(&attr, kern));
        launch_regs = attr.numRegs;
        launch_regs_cache.store(launch_regs, std::memory_order_relaxed);
    }
    if (launch_regs * fp4attn::kFwdThreads < 128 * fp4attn::kCtlRegs + 256 * fp4attn::kSmRegs ||
        launch_regs > fp4attn::kLaunchRegs)
        return fail(FP4ATTN_ECUDA, "attention kernel built with %d registers/thread; the register split needs %d",
                    launch_regs, fp4attn::kLaunchRegs);
    static std::atomic<unsigned long long> smem_set[kMaxDevices]{};
    if (int rc = set_smem_once(kern, C::SMEM_BYTES, smem_set)) return rc;
    if (slices > 65535) return fail(FP4ATTN_EINVAL, "batch*heads = %lld exceeds 65535", static_cast<long long>(slices));
    // Attention output is written by TMA stores in 32-row x OCH_E-column boxes
    // (the scores path stores from registers and ignores this map).
    CUtensorMap to = tq;
    fp4attn::FwdArgs pa = a;
    pa.scores_tma = 0;
    if constexpr (kScores) {
        // S [slices][seq_q][seq_k] FP32 leaves by TMA stores in 32-row x OCH_E
        // boxes when its rows are a whole number of 16-byte units.
        if (a.seq_k % 4 == 0) {
            const int rc = make_map_3d(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.out, a.seq_k, a.seq_q, slices,
                                       C::OCH_E, 32, swizzle_for(C::OCH_E * 4));
            if (rc) return rc;
            pa.scores_tma = 1;
        }
    } else {
        constexpr bool f32 = sizeof(OutT) == 4;
        const int rc = make_map_3d(&to, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                   static_cast<int>(sizeof(OutT)), a.out, D, a.seq_q, slices, C::OCH_E, 32,
                                   swizzle_for(C::OCH_E * static_cast<int>(sizeof(OutT))));
        if (rc) return rc;
    }
    // Persistent: one CTA per SM walks the (slice, query tile) items.
    const int64_t items = static_cast<int64_t>(a.nq_tiles) * slices;
    if (items > INT32_MAX) return fail(FP4ATTN_EINVAL, "too many query tiles");
    pa.n_items = static_cast<int>(items);
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(items, device_sms()));
    return launch_dependent(kern, grid, fp4attn::kFwdThreads, C::SMEM_BYTES, st, tq, tk, tv, to, pa);
}

// Share of the exponentials computed by the FMA-pipe polynomial, in eighths
// (FP4ATTN_POLY8 overrides it for the FP16-output D=128 kernel, for tuning).
int poly8_setting()
{
    static int v = [] {
        const char* s = getenv("FP4ATTN_POLY8");
        return s ? atoi(s) : -1;
    }();
    return v;
}

// Whether the paired kernel exponentiates against the running max while it
// forms the row max (FP4ATTN_SPEC=0 turns it off for the FP16-output D=128
// kernel, for comparison).
int spec_setting()
{
    static int v = [] {
        const char* s = getenv("FP4ATTN_SPEC");
        return s ? atoi(s) : -1;
    }();
    return v;
}

template <int D, int BN, typename OutT, bool kScores>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const fp4attn::FwdArgs& a,
               int64_t slices, cudaStream_t st)
{
    return launch_fwd_poly<D, BN, OutT, kScores, 3>(tq, tk, tv, a, slices, st);
}

template <int D, typename OutT, int kPoly8, bool kSpec, bool kSmall = false, bool kWithhold = false,
          bool kFuseQ = false, bool kLse = false>
int launch_pair_poly(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const fp4attn::FwdArgs& fa,
                     int64_t slices, cudaStream_t st)
{
    using C = fp4attn::PairCfg<D, kFuseQ ? 2 : 1>;
    auto kern = fp4attn::fp4_attention_pair_kernel<D, OutT, kPoly8, kSpec, kSmall, kWithhold, kFuseQ, kLse>;
    static std::atomic<int> launch_regs_cache{-1};
    int launch_regs = launch_regs_cache.load(std::memory_order_relaxed);
    if (launch_regs < 0) {
        cudaFuncAttributes attr;
        FP4_CUDA(cudaFuncGetAttributes(&attr, kern));
        launch_regs = attr.numRegs;
        launch_regs_cache.store(launch_regs, std::memory_order_relaxed);
    }
    if (launch_regs * fp4attn::kFwdThreads < 128 * fp4attn::PairRegs<kFuseQ>::kCtl + 256 * fp4attn::PairRegs<kFuseQ>::kSm ||
        launch_regs > fp4attn::kLaunchRegs)
        return fail(FP4ATTN_ECUDA, "attention kernel built with %d registers/thread; the register split needs %d",
                    launch_regs, fp4attn::kLaunchRegs);
    static std::atomic<unsigned long long> smem_set[kMaxDevices]{};
    if (int rc = set_smem_once(kern, C::SMEM_BYTES, smem_set)) return rc;
    if (slices > 65535) return fail(FP4ATTN_EINVAL, "batch*heads = %lld exceeds 65535", static_cast<long long>(slices));
    fp4attn::PairArgs a;
    a.seq_q = fa.seq_q;
    a.seq_k = fa.seq_k;
    a.nk_tiles = fa.nk_tiles;
    a.q_sf_tiles = fa.q_sf_tiles;
    a.scale_log2 = fa.scale_log2;
    a.out = fa.out;
    a.q_sf = fa.q_sf;
    a.k_sf = fa.k_sf;
    a.timeout_ns = fa.timeout_ns;
    a.causal = fa.causal;
    a.causal_off = fa.causal_off;
    a.qtiles = fa.qtiles;
    a.kparts = fa.kparts;
    a.nk_part = fa.nk_part;
    a.part_ml = fa.part_ml;
    a.part_o = fa.part_o;
    a.part_count = fa.part_count;
    a.q_in = static_cast<const __half*>(fa.q_in);
    a.ocp_mode = fa.ocp_mode;
    a.lse = fa.lse;
    // Output written by TMA stores in 32-row x 32-column boxes (64-byte rows
    // for FP16, 128-byte rows for FP32, swizzled to match the staging).
    CUtensorMap to;
    constexpr bool f32 = sizeof(OutT) == 4;
    int rc = make_map_3d(&to, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         static_cast<int>(sizeof(OutT)), fa.out, D, fa.seq_q, slices, 32, 32,
                         f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    // Key partitions: unnormalised FP32 O of every (item, tile) row, stored
    // by TMA in 32-row x 32-column boxes (128-byte rows, swizzled).
    CUtensorMap tp = to;
    if (fa.kparts > 1) {
        const uint64_t rows = static_cast<uint64_t>(slices) * fa.n_pairs * fa.kparts * fa.qtiles * 128;
        if ((rc = make_map_3d(&tp, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, fa.part_o, D, rows, 1, 32, 32,
                              CU_TENSOR_MAP_SWIZZLE_128B)))
            return rc;
    }
    // Persistent: one CTA per SM walks the (slice, query group, key partition) items.
    a.n_pairs = fa.n_pairs;
    const int64_t items = static_cast<int64_t>(a.n_pairs) * slices * fa.kparts;
    if (items > INT32_MAX) return fail(FP4ATTN_EINVAL, "too many query tiles");
    a.n_items = static_cast<int>(items);
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(items, device_sms()));
    return launch_dependent(kern, grid, fp4attn::kFwdThreads, C::SMEM_BYTES, st, tq, tk, tv, to, tp, a);
}

template <int D, typename OutT>
int launch_pair(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const fp4attn::FwdArgs& a,
                int64_t slices, cudaStream_t st)
{
    // The forward that also writes the log-sum-exp rows (the backward pass's
    // head dims: all of this kernel's).
    {
        if (a.lse) {
            if (a.qtiles == 1 || a.kparts > 1)
                return launch_pair_poly<D, OutT, 3, true, true, false, false, true>(tq, tk, tv, a, slices, st);
            return launch_pair_poly<D, OutT, 3, true, false, false, false, true>(tq, tk, tv, a, slices, st);
        }
    }
    // Q quantised inside the attention kernel (the large-problem schedule).
    if (a.q_in) return launch_pair_poly<D, OutT, 3, true, false, false, true>(tq, tk, tv, a, slices, st);
    // One query tile per item or key partitions: the small-problem kernel.
    if (a.qtiles == 1 || a.kparts > 1) return launch_pair_poly<D, OutT, 3, true, true>(tq, tk, tv, a, slices, st);
    if constexpr (D == 128 && sizeof(OutT) == 2) {
        const bool spec = spec_setting() != 0;
        switch (poly8_setting()) {
            case 2: return spec ? launch_pair_poly<D, OutT, 2, true>(tq, tk, tv, a, slices, st)
                                : launch_pair_poly<D, OutT, 2, false>(tq, tk, tv, a, slices, st);
            case 4: return spec ? launch_pair_poly<D, OutT, 4, true>(tq, tk, tv, a, slices, st)
                                : launch_pair_poly<D, OutT, 4, false>(tq, tk, tv, a, slices, st);
            default:
                if (!spec) return launch_pair_poly<D, OutT, 3, false>(tq, tk, tv, a, slices, st);
                break;
        }
    }
    return launch_pair_poly<D, OutT, 3, true>(tq, tk, tv, a, slices, st);
}

template <int D, bool kScores>
int dispatch_out(int out_dtype, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const fp4attn::FwdArgs& a, int64_t slices, cudaStream_t st)
{
    constexpr int BN = D == 160 ? 128 : 64;
    if constexpr (kScores) {
        return launch_fwd<D, BN, float, true>(tq, tk, tv, a, slices, st);
    } else if constexpr (D <= 128) {
        if (out_dtype == FP4ATTN_F32) return launch_pair<D, float>(tq, tk, tv, a, slices, st);
        return launch_pair<D, __half>(tq, tk, tv, a, slices, st);
    } else {
        if (out_dtype == FP4ATTN_F32) return launch_fwd<D, BN, float, false>(tq, tk, tv, a, slices, st);
        return launch_fwd<D, BN, __half, false>(tq, tk, tv, a, slices, st);
    }
}

template <bool kScores>
int dispatch_dim(int d, int out_dtype, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                 const fp4attn::FwdArgs& a, int64_t slices, cudaStream_t st)
{
    switch (d) {
        case 32: return dispatch_out<32, kScores>(out_dtype, tq, tk, tv, a, slices, st);
        case 64: return dispatch_out<64, kScores>(out_dtype, tq, tk, tv, a, slices, st);
        case 96: return dispatch_out<96, kScores>(out_dtype, tq, tk, tv, a, slices, st);
        case 128: return dispatch_out<128, kScores>(out_dtype, tq, tk, tv, a, slices, st);
        case 160: return dispatch_out<160, kScores>(out_dtype, tq, tk, tv, a, slices, st);
        case 256: return dispatch_out<256, kScores>(out_dtype, tq, tk, tv, a, slices, st);
    }
    return fail(FP4ATTN_EUNSUPPORTED, "head_dim %d not compiled", d);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_problem(const void* Q, const void* K, const void* V, const void* Out, int in_dtype, int out_dtype, int batch,
                  int heads, int sq, int sk, int d, int scale_mode, bool need_v)
{
    if (!Q || !K || !Out || (need_v && !V)) return fail(FP4ATTN_EINVAL, "null tensor pointer");
    if (!aligned16(Q) || !aligned16(K) || !aligned16(Out) || (need_v && !aligned16(V)))
        return fail(FP4ATTN_EINVAL, "tensor pointers must be 16-byte aligned");
    if (in_dtype != FP4ATTN_F32 && in_dtype != FP4ATTN_F16) return fail(FP4ATTN_EINVAL, "in_dtype %d", in_dtype);
    if (out_dtype != FP4ATTN_F32 && out_dtype != FP4ATTN_F16) return fail(FP4ATTN_EINVAL, "out_dtype %d", out_dtype);
    if (scale_mode != FP4ATTN_SCALE_REFERENCE && scale_mode != FP4ATTN_SCALE_OCP)
        return fail(FP4ATTN_EINVAL, "scale_mode %d", scale_mode);
    if (batch < 1 || heads < 1 || sq < 1 || sk < 1)
        return fail(FP4ATTN_EINVAL, "batch, heads, seq_q and seq_k must be >= 1 (got %d, %d, %d, %d)", batch, heads, sq,
                    sk);
    if (!supported_dim(d)) return fail(FP4ATTN_EUNSUPPORTED, "head_dim %d is not one of 32/64/96/128/160/256", d);
    if (static_cast<int64_t>(batch) * heads > 65535) return fail(FP4ATTN_EINVAL, "batch*heads exceeds 65535");
    return FP4ATTN_OK;
}

struct Problem {
    int64_t slices;
    int sq, sk, d;
    Workspace w;
};

int check_workspace(const Problem& p, const void* workspace, size_t ws_bytes)
{
    if (!workspace || ws_bytes < p.w.total)
        return fail(FP4ATTN_EWORKSPACE, "workspace of %zu bytes needed, %zu given", p.w.total, workspace ? ws_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail(FP4ATTN_EINVAL, "workspace must be 256-byte aligned");
    return FP4ATTN_OK;
}

// q_slices >= 0: quantise Q of the first q_slices slices only (the rest is
// quantised by the attention kernel itself, fp4attn_forward_fused_q).
int do_prepare(const void* Q, const void* K, const void* V, int in_dtype, int batch, int heads, int sq, int sk, int d,
               int scale_mode, void* workspace, size_t ws_bytes, void* stream, bool need_v, int64_t q_slices = -1)
{
    int rc = check_problem(Q, K, V, Q, in_dtype, FP4ATTN_F32, batch, heads, sq, sk, d, scale_mode, need_v);
    if (rc) return rc;
    if ((rc = device_ready())) return rc;
    Problem p{static_cast<int64_t>(batch) * heads, sq, sk, d, {}};
    p.w = plan_workspace(p.slices, sq, sk, d, need_v ? in_dtype : FP4ATTN_F16);
    if ((rc = check_workspace(p, workspace, ws_bytes))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int bn = block_n_for(d);
    const int nq_sf = q_sf_tiles(sq, d), nk_sf = (sk + bn - 1) / bn;
    const int ocp = scale_mode == FP4ATTN_SCALE_OCP;
    const fp4attn::QuantJob jq{Q, ws + p.w.q_codes, ws + p.w.q_sf,
                               quant_args(q_slices >= 0 ? std::min(q_slices, p.slices) : p.slices, sq, d, 128, nq_sf,
                                          ocp)};
    const fp4attn::QuantJob jk{K, ws + p.w.k_codes, ws + p.w.k_sf, quant_args(p.slices, sk, d, bn, nk_sf, ocp)};
    // The attention kernel's key-partition arrival counters start at zero (it
    // leaves them at zero when it completes).
    const int n_zero = static_cast<int>((p.w.part_count == p.w.total ? 0 : p.w.total - p.w.part_count) / 4);
    uint32_t* zero = reinterpret_cast<uint32_t*>(ws + p.w.part_count);
    if (in_dtype == FP4ATTN_F16 || !need_v) {
        const fp4attn::VConvJob jv{nullptr, nullptr, 0, zero, n_zero};
        if (in_dtype == FP4ATTN_F16) rc = launch_quant_qk<__half>(jq, jk, &jv, p.slices, st);
        else rc = launch_quant_qk<float>(jq, jk, &jv, p.slices, st);
        if (rc) return rc;
    } else {
        const fp4attn::VConvJob jv{static_cast<const float4*>(V), reinterpret_cast<uint2*>(ws + p.w.v16),
                                   static_cast<int64_t>(sk) * d / 4, zero, n_zero};
        if ((rc = launch_quant_qk<float>(jq, jk, &jv, p.slices, st))) return rc;
    }
    return FP4ATTN_OK;
}

// test_timeout_ns > 0: the abort self-test (fp4attn_selftest_abort) -- the
// head_dim 64, FP32-output pair kernel with one withheld arrival, waits
// bounded by test_timeout_ns.
int do_attend(const void* V, void* Out, int in_dtype, int out_dtype, int batch, int heads, int sq, int sk, int d,
              float softmax_scale, const void* workspace, size_t ws_bytes, void* stream, bool scores,
              int mask_mode = FP4ATTN_MASK_NONE, unsigned long long test_timeout_ns = 0, const void* q_in = nullptr,
              int ocp_mode = 0, float* lse = nullptr)
{
    if (mask_mode != FP4ATTN_MASK_NONE && mask_mode != FP4ATTN_MASK_CAUSAL)
        return fail(FP4ATTN_EINVAL, "mask_mode %d", mask_mode);
    const void* dummy = workspace;
    int rc = check_problem(dummy, dummy, V, Out, in_dtype, out_dtype, batch, heads, sq, sk, d, FP4ATTN_SCALE_REFERENCE,
                           !scores);
    if (rc) return rc;
    if ((rc = device_ready())) return rc;
    Problem p{static_cast<int64_t>(batch) * heads, sq, sk, d, {}};
    p.w = plan_workspace(p.slices, sq, sk, d, scores ? FP4ATTN_F16 : in_dtype);
    if ((rc = check_workspace(p, workspace, ws_bytes))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint8_t* ws = static_cast<const uint8_t*>(workspace);
    const int dp = padded_dim(d), bn = block_n_for(d);
    const int cw = dp / 2 == 96 ? 32 : dp / 2;
    CUtensorMap tq, tk, tv;
    if ((rc = make_map_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + p.w.q_codes, dp / 2, sq, p.slices, cw, 128,
                          swizzle_for(cw))))
        return rc;
    if ((rc = make_map_3d(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + p.w.k_codes, dp / 2, sk, p.slices, cw, bn,
                          swizzle_for(cw))))
        return rc;
    tv = tk;
    if (!scores) {
        const void* v16 = in_dtype == FP4ATTN_F32 ? static_cast<const void*>(ws + p.w.v16) : V;
        // The V chunk width of the kernel that runs (PairCfg / FwdCfg::VCW).
        const int vcw = paired(d) ? ((2 * d) % 128 == 0 ? 128 : 64) : 128;
        if ((rc = make_map_3d(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, v16, d, sk, p.slices, vcw / 2, bn,
                              swizzle_for(vcw))))
            return rc;
    }
    fp4attn::FwdArgs a;
    a.seq_q = sq;
    a.seq_k = sk;
    a.nq_tiles = (sq + 127) / 128;
    a.q_sf_tiles = q_sf_tiles(sq, d);
    a.nk_tiles = (sk + bn - 1) / bn;
    const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(static_cast<float>(d));
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = Out;
    a.q_sf = ws + p.w.q_sf;
    a.k_sf = ws + p.w.k_sf;
    a.timeout_ns = wait_timeout_ns();
    a.causal = mask_mode == FP4ATTN_MASK_CAUSAL ? 1 : 0;
    a.causal_off = sk - sq;
    {
        const PairPlan pp = pair_plan(p.slices, sq, sk, d, a.causal != 0);
        a.qtiles = pp.qtiles;
        a.n_pairs = pp.n_pairs;
        a.kparts = paired(d) ? pp.kparts : 1;
        a.nk_part = pp.nk_part;
        a.part_o = reinterpret_cast<float*>(const_cast<uint8_t*>(ws) + p.w.part_o);
        a.part_ml = reinterpret_cast<float2*>(const_cast<uint8_t*>(ws) + p.w.part_ml);
        a.part_count = reinterpret_cast<unsigned*>(const_cast<uint8_t*>(ws) + p.w.part_count);
    }
    a.q_in = q_in;
    a.ocp_mode = ocp_mode;
    a.lse = lse;
    if (lse && !paired(d))
        return fail(FP4ATTN_EUNSUPPORTED, "the log-sum-exp output covers head_dim 32 to 128 (got %d)", d);
    if (scores) return dispatch_dim<true>(d, FP4ATTN_F32, tq, tk, tv, a, p.slices, st);
    if (test_timeout_ns) {
        if (d != 64 || out_dtype != FP4ATTN_F32 || a.qtiles != 2 || a.kparts != 1 || a.causal)
            return fail(FP4ATTN_EINVAL, "the abort self-test runs head_dim 64, FP32 output, seq_q > 128, no key "
                                        "partitions, no mask");
        a.timeout_ns = test_timeout_ns;
        return launch_pair_poly<64, float, 3, true, false, true>(tq, tk, tv, a, p.slices, st);
    }
    return dispatch_dim<false>(d, out_dtype, tq, tk, tv, a, p.slices, st);
}

}  // namespace

namespace fp4attn {
// Lets other translation units of the library report a detail through
// fp4attn_last_error().
void set_error_detail(const char* msg) { g_last_error = msg; }

// The host helpers above, for the library's other translation units
// (backward.cu).
namespace host {
int error(int code, const char* msg) { return fail(code, "%s", msg); }
int ready() { return device_ready(); }
int sms() { return device_sms(); }
unsigned long long timeout_ns() { return wait_timeout_ns(); }
int map3d(CUtensorMap* m, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t inner, uint64_t rows,
          uint64_t slices, uint32_t box_inner, uint32_t box_rows, int swizzle_bytes)
{
    return make_map_3d(m, dt, elem_bytes, base, inner, rows, slices, box_inner, box_rows, swizzle_for(swizzle_bytes));
}
}  // namespace host
}  // namespace fp4attn

extern "C" {

int fp4attn_quantize(const void* x, int dtype, int64_t rows, int head_dim, uint8_t* codes, uint8_t* scales,
                     int scale_mode, int layout, void* stream)
{
    g_last_error.clear();
    if (rows == 0 && head_dim >= 32 && head_dim % 32 == 0) return FP4ATTN_OK;
    if (!x || !codes || !scales) return fail(FP4ATTN_EINVAL, "null pointer");
    if (!aligned16(x) || !aligned16(codes)) return fail(FP4ATTN_EINVAL, "x and codes must be 16-byte aligned");
    if (rows < 0 || head_dim < 32 || head_dim % 32) return fail(FP4ATTN_EINVAL, "rows >= 0, head_dim a multiple of 32");
    if (dtype != FP4ATTN_F32 && dtype != FP4ATTN_F16) return fail(FP4ATTN_EINVAL, "dtype %d", dtype);
    if (scale_mode != FP4ATTN_SCALE_REFERENCE && scale_mode != FP4ATTN_SCALE_OCP)
        return fail(FP4ATTN_EINVAL, "scale_mode %d", scale_mode);
    if (layout != FP4ATTN_LAYOUT_ROWMAJOR) return fail(FP4ATTN_EINVAL, "layout %d", layout);
    int rc = device_ready();
    if (rc) return rc;
    if (rows == 0) return FP4ATTN_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t work = rows * (head_dim / 32);
    const int ocp = scale_mode == FP4ATTN_SCALE_OCP;
    if (dtype == FP4ATTN_F16)
        fp4attn::quantize_rowmajor_kernel<__half>
            <<<grid_for(work), 256, 0, st>>>(static_cast<const __half*>(x), rows, head_dim, codes, scales, ocp);
    else
        fp4attn::quantize_rowmajor_kernel<float>
            <<<grid_for(work), 256, 0, st>>>(static_cast<const float*>(x), rows, head_dim, codes, scales, ocp);
    FP4_CUDA(cudaGetLastError());
    return FP4ATTN_OK;
}

size_t fp4attn_workspace_size(int batch, int heads, int seq_q, int seq_k, int head_dim, int in_dtype)
{
    if (batch < 1 || heads < 1 || seq_q < 1 || seq_k < 1 || !supported_dim(head_dim)) return 0;
    if (in_dtype != FP4ATTN_F32 && in_dtype != FP4ATTN_F16) return 0;
    return plan_workspace(static_cast<int64_t>(batch) * heads, seq_q, seq_k, head_dim, in_dtype).total;
}

int fp4attn_prepare(const void* Q, const void* K, const void* V, int in_dtype, int batch, int heads, int seq_q,
                    int seq_k, int head_dim, int scale_mode, void* workspace, size_t workspace_bytes, void* stream)
{
    g_last_error.clear();
    return do_prepare(Q, K, V, in_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, workspace, workspace_bytes,
                      stream, true);
}

int fp4attn_attend(const void* V, void* Out, int in_dtype, int out_dtype, int batch, int heads, int seq_q, int seq_k,
                   int head_dim, float softmax_scale, const void* workspace, size_t workspace_bytes, void* stream)
{
    g_last_error.clear();
    return do_attend(V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale, workspace,
                     workspace_bytes, stream, false);
}

int fp4attn_forward(const void* Q, const void* K, const void* V, void* Out, int in_dtype, int out_dtype, int batch,
                    int heads, int seq_q, int seq_k, int head_dim, float softmax_scale, int scale_mode,
                    void* workspace, size_t workspace_bytes, void* stream)
{
    g_last_error.clear();
    int rc = check_problem(Q, K, V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, true);
    if (rc) return rc;
    if ((rc = do_prepare(Q, K, V, in_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, workspace,
                         workspace_bytes, stream, true)))
        return rc;
    return do_attend(V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale, workspace,
                     workspace_bytes, stream, false);
}

int fp4attn_forward_fused_q(const void* Q, const void* K, const void* V, void* Out, int in_dtype, int out_dtype,
                            int batch, int heads, int seq_q, int seq_k, int head_dim, float softmax_scale,
                            int scale_mode, void* workspace, size_t workspace_bytes, void* stream)
{
    g_last_error.clear();
    int rc = check_problem(Q, K, V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, true);
    if (rc) return rc;
    const PairPlan pp = pair_plan(static_cast<int64_t>(batch) * heads, seq_q, seq_k, head_dim, false);
    // Warp 3 quantises one item's 256 query rows while the item before it
    // runs; with fewer than kFusedQMinKeyTiles 64-key steps per item it would
    // hold the kernel up, so shorter key ranges keep the pre-pass.
    constexpr int kFusedQMinKeyTiles = 48;
    if (in_dtype != FP4ATTN_F16 || !paired(head_dim) || pp.qtiles != 2 || pp.kparts != 1 ||
        (seq_k + 63) / 64 < kFusedQMinKeyTiles)
        // Outside the in-kernel quantiser's scope: the two-launch path (same result).
        return fp4attn_forward(Q, K, V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale,
                               scale_mode, workspace, workspace_bytes, stream);
    // The pre-pass quantises the Q rows of each CTA's first work item (items
    // 0 .. grid-1 of the persistent schedule, the leading slices); the kernel
    // quantises every later item's Q while the item before it runs.
    if ((rc = device_ready())) return rc;
    const int64_t grid = std::min<int64_t>(pp.groups, device_sms());
    const int64_t q_slices = (grid + pp.n_pairs - 1) / pp.n_pairs;
    if ((rc = do_prepare(Q, K, V, in_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, workspace,
                         workspace_bytes, stream, true, q_slices)))
        return rc;
    return do_attend(V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale, workspace,
                     workspace_bytes, stream, false, FP4ATTN_MASK_NONE, 0, Q, scale_mode == FP4ATTN_SCALE_OCP);
}

int fp4attn_attend_masked(const void* V, void* Out, int in_dtype, int out_dtype, int batch, int heads, int seq_q,
                          int seq_k, int head_dim, float softmax_scale, int mask_mode, const void* workspace,
                          size_t workspace_bytes, void* stream)
{
    g_last_error.clear();
    return do_attend(V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale, workspace,
                     workspace_bytes, stream, false, mask_mode);
}

int fp4attn_forward_masked(const void* Q, const void* K, const void* V, void* Out, int in_dtype, int out_dtype,
                           int batch, int heads, int seq_q, int seq_k, int head_dim, float softmax_scale,
                           int scale_mode, int mask_mode, void* workspace, size_t workspace_bytes, void* stream)
{
    g_last_error.clear();
    if (mask_mode != FP4ATTN_MASK_NONE && mask_mode != FP4ATTN_MASK_CAUSAL)
        return fail(FP4ATTN_EINVAL, "mask_mode %d", mask_mode);
    int rc = check_problem(Q, K, V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, true);
    if (rc) return rc;
    if ((rc = do_prepare(Q, K, V, in_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, workspace,
                         workspace_bytes, stream, true)))
        return rc;
    return do_attend(V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale, workspace,
                     workspace_bytes, stream, false, mask_mode);
}

int fp4attn_forward_lse(const void* Q, const void* K, const void* V, void* Out, float* lse, int in_dtype,
                        int out_dtype, int batch, int heads, int seq_q, int seq_k, int head_dim, float softmax_scale,
                        int scale_mode, int mask_mode, void* workspace, size_t workspace_bytes, void* stream)
{
    g_last_error.clear();
    if (mask_mode != FP4ATTN_MASK_NONE && mask_mode != FP4ATTN_MASK_CAUSAL)
        return fail(FP4ATTN_EINVAL, "mask_mode %d", mask_mode);
    if (!lse || (reinterpret_cast<uintptr_t>(lse) & 3u)) return fail(FP4ATTN_EINVAL, "lse must be a 4-byte aligned pointer");
    int rc = check_problem(Q, K, V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, true);
    if (rc) return rc;
    if (!paired(head_dim))
        return fail(FP4ATTN_EUNSUPPORTED, "the log-sum-exp output covers head_dim 32 to 128 (got %d)", head_dim);
    if ((rc = do_prepare(Q, K, V, in_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, workspace,
                         workspace_bytes, stream, true)))
        return rc;
    return do_attend(V, Out, in_dtype, out_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale, workspace,
                     workspace_bytes, stream, false, mask_mode, 0, nullptr, 0, lse);
}

int fp4attn_debug_scores(const void* Q, const void* K, float* S, int in_dtype, int batch, int heads, int seq_q,
                         int seq_k, int head_dim, int scale_mode, void* workspace, size_t workspace_bytes,
                         void* stream)
{
    g_last_error.clear();
    int rc = check_problem(Q, K, nullptr, S, in_dtype, FP4ATTN_F32, batch, heads, seq_q, seq_k, head_dim, scale_mode,
                           false);
    if (rc) return rc;
    if ((rc = do_prepare(Q, K, nullptr, in_dtype, batch, heads, seq_q, seq_k, head_dim, scale_mode, workspace,
                         workspace_bytes, stream, false)))
        return rc;
    return do_attend(nullptr, S, in_dtype, FP4ATTN_F32, batch, heads, seq_q, seq_k, head_dim, 1.0f, workspace,
                     workspace_bytes, stream, true);
}

int fp4attn_status_query(void* stream)
{
    g_last_error.clear();
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    FP4_CUDA(cudaStreamSynchronize(st));
    int host[4] = {0, 0, 0, 0};
    FP4_CUDA(cudaMemcpyFromSymbol(host, fp4attn::g_fp4attn_error, sizeof host));
    if (host[0] == 0) return FP4ATTN_OK;
    const int zero[4] = {0, 0, 0, 0};
    FP4_CUDA(cudaMemcpyToSymbol(fp4attn::g_fp4attn_error, zero, sizeof zero));
    return fail(host[0], "device wait expired at site %d (block %d,%d)", host[1], host[2], host[3]);
}

int fp4attn_selftest_timeout(unsigned timeout_us, void* stream)
{
    g_last_error.clear();
    int rc = device_ready();
    if (rc) return rc;
    if (timeout_us < 1 || timeout_us > 10000000u) return fail(FP4ATTN_EINVAL, "timeout_us in [1, 1e7]");
    fp4attn::timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<unsigned long long>(timeout_us) * 1000ull);
    FP4_CUDA(cudaGetLastError());
    return FP4ATTN_OK;
}

int fp4attn_selftest_abort(const void* V, void* Out, int batch, int heads, int seq_q, int seq_k,
                           const void* workspace, size_t workspace_bytes, unsigned timeout_us, void* stream)
{
    g_last_error.clear();
    if (timeout_us < 1 || timeout_us > 10000000u) return fail(FP4ATTN_EINVAL, "timeout_us in [1, 1e7]");
    return do_attend(V, Out, FP4ATTN_F16, FP4ATTN_F32, batch, heads, seq_q, seq_k, 64, 0.f, workspace,
                     workspace_bytes, stream, false, FP4ATTN_MASK_NONE, static_cast<unsigned long long>(timeout_us) * 1000ull);
}

int fp4attn_selftest_exp2(const float* x, float* y, int64_t n, void* stream)
{
    g_last_error.clear();
    int rc = device_ready();
    if (rc) return rc;
    if (n < 0 || n % 2 || (n && (!x || !y)) || !aligned16(x) || !aligned16(y))
        return fail(FP4ATTN_EINVAL, "n must be even and >= 0, x and y 16-byte aligned");
    if (n == 0) return FP4ATTN_OK;
    fp4attn::exp2_poly_selftest_kernel<<<grid_for(n / 2), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const float2*>(x), reinterpret_cast<float2*>(y), n / 2);
    FP4_CUDA(cudaGetLastError());
    return FP4ATTN_OK;
}

const char* fp4attn_error_string(int status)
{
    switch (status) {
        case FP4ATTN_OK: return "ok";
        case FP4ATTN_EINVAL: return "invalid argument";
        case FP4ATTN_EUNSUPPORTED: return "unsupported head_dim or device";
        case FP4ATTN_ECUDA: return "CUDA error";
        case FP4ATTN_ETIMEOUT: return "device wait timed out";
        case FP4ATTN_EWORKSPACE: return "workspace missing or too small";
    }
    return "unknown status";
}

const char* fp4attn_last_error(void) { return g_last_error.c_str(); }

int fp4attn_supported_head_dims(int* dims, int cap)
{
    int n = 0;
    for (int x : kSupportedDims) {
        if (dims && n < cap) dims[n] = x;
        n++;
    }
    return n;
}

}  // extern "C"

// The backward pass (its kernels and C entry points) in this translation unit.
#include "backward_api.cuh"
