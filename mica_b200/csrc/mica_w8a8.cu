// mica_w8a8.cu -- the single translation unit of libmica_w8a8.so: kernels (included
// headers) and the extern "C" entry points declared in include/mica_w8a8.h.
//
// Host side: argument and alignment checks that return status codes (the reference's
// launcher turns the same conditions into `None` misses, v0.5/serving/lib/
// int8_kernels.py:268-311, :325-406), TMA descriptor encoding, tile choice and launch.
#include <type_traits>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "gemm_i8.cuh"
#include "gemm_i8_pair.cuh"
#include "gemm_i8_splitk.cuh"
#include "gemm_i8_streamk.cuh"
#include "quant.cuh"
#include "readout.cuh"
#include "qk_rope.cuh"
#include "attention.cuh"

using namespace mica;

// ======================================================================================
// host helpers
// ======================================================================================
namespace mica_host {

static thread_local char t_err[256] = {0};

void set_cuda_error(cudaError_t e) {
    snprintf(t_err, sizeof(t_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr int kMaxDev = 64;
struct DevInfo {
    std::atomic<int> state{0};  // 0 unknown, 1 ok, 2 unsupported
    int sm_count = 0;
    int smem_optin = 0;
};
static DevInfo g_dev[kMaxDev];
static std::mutex g_lock;

int check_device(int* sm_count) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    if (dev < 0 || dev >= kMaxDev) return MICA_ERR_ARCH;
    DevInfo& d = g_dev[dev];
    int st = d.state.load(std::memory_order_acquire);
    if (st == 0) {
        std::lock_guard<std::mutex> g(g_lock);
        st = d.state.load(std::memory_order_relaxed);
        if (st == 0) {
            int major = 0, minor = 0, sms = 0, optin = 0;
            if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
                (e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
                (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
                (e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) {
                set_cuda_error(e);
                return MICA_ERR_CUDA;
            }
            d.sm_count = sms;
            d.smem_optin = optin;
            // sm_100a code runs on compute capability 10.0 only.
            st = (major == 10 && minor == 0 && optin >= 232448) ? 1 : 2;
            d.state.store(st, std::memory_order_release);
        }
    }
    if (st != 1) return MICA_ERR_ARCH;
    if (sm_count) *sm_count = d.sm_count;
    return MICA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) {
        snprintf(t_err, sizeof(t_err), "cuTensorMapEncodeTiled entry point not found");
        return MICA_ERR_CUDA;
    }
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(t_err, sizeof(t_err), "cuTensorMapEncodeTiled failed: CUresult %d", static_cast<int>(r));
        return MICA_ERR_CUDA;
    }
    return MICA_OK;
}

static int launch_status() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    return MICA_OK;
}

static size_t dt_size(int dt) { return dt == MICA_DT_FP32 ? 4 : 2; }

// ---- GEMM kernel registry ------------------------------------------------------------
template <int BN, int EPI, typename OutT, int EW = 4>
static int gemm_prepare() {
    int dev = 0;
    cudaGetDevice(&dev);
    static std::atomic<uint64_t> done{0};  // one bit per device
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return MICA_OK;
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel<BN, EPI, OutT, EW>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, GemmShape<BN, EW>::SMEM_BYTES);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    done.fetch_or(bit, std::memory_order_release);
    return MICA_OK;
}

template <int BN, int EPI, typename OutT, int EW = 4>
static int gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& args,
                       int grid, bool cooperative, cudaStream_t stream) {
    int rc = gemm_prepare<BN, EPI, OutT, EW>();
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GemmShape<BN, EW>::THREADS);
    cfg.dynamicSmemBytes = GemmShape<BN, EW>::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (cooperative) {
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_i8_kernel<BN, EPI, OutT, EW>, ta, tb, tc, args);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    return launch_status();
}

// Epilogue warps of the dequant GEMM per tile width. The 320-wide tile runs one tile per CTA, so
// nothing hides its epilogue: eight warps (two per tensor-memory lane quarter) halve it.
template <int BN>
struct DequantWarps { static constexpr int EW = BN == 320 ? 8 : 4; };

// ---- CTA-pair kernels ---------------------------------------------------------------------
// Co-resident clusters of two per device (pairs of SMs the scheduler can place together).
static std::atomic<int> g_pair_clusters[kMaxDev];

template <int BN, typename OutT>
static int pair_prepare(int* max_clusters) {
    int dev = 0;
    cudaGetDevice(&dev);
    static std::atomic<uint64_t> done{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(done.load(std::memory_order_acquire) & bit)) {
        cudaError_t e = cudaFuncSetAttribute(gemm_i8_pair_kernel<BN, OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             PairShape<BN>::SMEM_BYTES);
        if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
        if (g_pair_clusters[dev].load() == 0) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * 512);
            cfg.blockDim = dim3(PairShape<BN>::THREADS);
            cfg.dynamicSmemBytes = PairShape<BN>::SMEM_BYTES;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 2;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            e = cudaOccupancyMaxActiveClusters(&n, gemm_i8_pair_kernel<BN, OutT>, &cfg);
            if (e != cudaSuccess || n < 1) {
                set_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidConfiguration);
                return MICA_ERR_CUDA;
            }
            g_pair_clusters[dev].store(n);
        }
        done.fetch_or(bit, std::memory_order_release);
    }
    *max_clusters = g_pair_clusters[dev].load();
    return MICA_OK;
}

template <int BN, typename OutT>
static int pair_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& args,
                       long tiles, int max_ctas, cudaStream_t stream) {
    int clusters = 0;
    int rc = pair_prepare<BN, OutT>(&clusters);
    if (rc) return rc;
    if (max_ctas > 0 && clusters > max_ctas / 2) clusters = max_ctas / 2 > 0 ? max_ctas / 2 : 1;
    if (tiles < clusters) clusters = static_cast<int>(tiles);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(PairShape<BN>::THREADS);
    cfg.dynamicSmemBytes = PairShape<BN>::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_i8_pair_kernel<BN, OutT>, ta, tb, tc, args);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    return launch_status();
}

// Tile choice when the caller (or the pinned table in the Python layer) gives none,
// from the measured sweep over the 4B model's projection shapes: the single-CTA 128 x 256
// tile wins whenever it fills a wave of SMs; below that 128 x 128, then 128 x 64.
// ---- split-K clusters ----------------------------------------------------------------
// Co-resident clusters of S split-K CTAs, per device, per tile width and S (0 = not queried).
static std::atomic<int> g_splitk_clusters[kMaxDev][3][9];

static int bn_index(int bn) { return bn == 256 ? 2 : (bn == 128 ? 1 : 0); }

template <int BN, typename OutT>
static int splitk_prepare(int dev) {
    static std::atomic<uint64_t> done{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return MICA_OK;
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_splitk_kernel<BN, OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GemmShape<BN, 4>::SMEM_BYTES);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    for (int s = 2; s <= 8; ++s) {
        if (g_splitk_clusters[dev][bn_index(BN)][s].load() != 0) continue;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(s * 64);
        cfg.blockDim = dim3(GemmShape<BN, 4>::THREADS);
        cfg.dynamicSmemBytes = GemmShape<BN, 4>::SMEM_BYTES;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = s;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, gemm_i8_splitk_kernel<BN, OutT>, &cfg);
        if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
        g_splitk_clusters[dev][bn_index(BN)][s].store(n > 0 ? n : -1);
    }
    done.fetch_or(bit, std::memory_order_release);
    return MICA_OK;
}

// The split factor for `tiles` output tiles of `num_kb` k-blocks: 1 (no split) unless fewer
// than half the SMs would get a tile; then the largest S <= 8 whose clusters are all
// co-resident, that keeps at least four k-blocks per rank, and leaves no rank empty.
static int choose_splits(int dev, int bn, long tiles, int num_kb, int sms) {
    if (2 * tiles > sms) return 1;
    for (int s = 8; s >= 2; --s) {
        const int co = g_splitk_clusters[dev][bn_index(bn)][s].load();
        const int per = (num_kb + s - 1) / s;
        if (co > 0 && tiles <= co && per >= 4 && (s - 1) * per < num_kb) return s;
    }
    return 1;
}

template <int BN, typename OutT>
static int splitk_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& args,
                         long tiles, int splits, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles * splits));
    cfg.blockDim = dim3(GemmShape<BN, 4>::THREADS);
    cfg.dynamicSmemBytes = GemmShape<BN, 4>::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_i8_splitk_kernel<BN, OutT>, ta, tb, tc, args);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    return launch_status();
}

template <int BN>
static int splitk_prepare_all(int dev) {
    int rc;
    if ((rc = splitk_prepare<BN, __nv_bfloat16>(dev)) || (rc = splitk_prepare<BN, __half>(dev)) ||
        (rc = splitk_prepare<BN, float>(dev)))
        return rc;
    return MICA_OK;
}

template <int BN>
static int splitk_dispatch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& g,
                           int c_dtype, long tiles, int splits, cudaStream_t st) {
    if (c_dtype == MICA_DT_BF16) return splitk_launch<BN, __nv_bfloat16>(ta, tb, tc, g, tiles, splits, st);
    if (c_dtype == MICA_DT_FP16) return splitk_launch<BN, __half>(ta, tb, tc, g, tiles, splits, st);
    return splitk_launch<BN, float>(ta, tb, tc, g, tiles, splits, st);
}

static void pick_tile(int M, int N, int sms, int* bm, int* bn) {
    const long m_blocks = (M + 127) / 128;
    const long t256 = m_blocks * ((N + 255) / 256);
    const long t128 = m_blocks * ((N + 127) / 128);
    const long t320 = m_blocks * ((N + 319) / 320);
    *bm = 128;
    *bn = t256 >= sms ? 256 : (2 * t128 >= sms ? 128 : 64);
    // A grid of 128 x 256 tiles just past one wave (config 0: 152 tiles on 148 SMs) leaves its
    // critical path at two tiles; 128 x 320 tiles fit one wave, each 1.25 tiles long.
    if (t256 > sms && t256 < 2L * sms && t320 <= sms) *bn = 320;
}

// ---- stream-K kernels ---------------------------------------------------------------------
// The library choice uses stream-K only for a grid of one to two waves whose second wave is
// long and mostly empty. On B200 the exchange of a cut tile costs about 6 us at the end of the
// kernel (the finishing CTA of a short last segment waits for its neighbour's partial), the
// flag clear about 2 us, and a run of many waves loses the round-robin order's L2 reuse, so
// the data-parallel kernel wins unless the critical path drops by SK_MIN_GAIN_KB k-blocks or
// more (measured: M 2048, N 2560, K 9728 at 128 x 256 goes from 69.6 to 57.4 us; M 512, N 9728,
// K 2560 rises from 28.7 to 32.9 us, and M 32768, N 2560, K 9728 from 582 to 713 us). It is
// weighed only for 128- and 256-wide tiles: where pick_tile takes 128 x 320 tiles (the grid then
// fits one wave) those win (55.3 us on the first shape above), so stream-K serves grids that
// 128 x 320 tiles cannot fit in one wave (M 2048, N 3072, K 9728: 71.7 -> 65.6 us).
constexpr long SK_MIN_GAIN_KB = 40;

static bool want_streamk(long tiles, int num_kb, int sms) {
    if (tiles < sms || tiles >= 2L * sms || sms > 256) return false;
    const long dp = 2L * num_kb;
    const long sk = (tiles * num_kb + sms - 1) / sms;
    return dp - sk >= SK_MIN_GAIN_KB;
}

static size_t streamk_ws_bytes(int ctas, int bn) {
    return static_cast<size_t>(SK_FLAG_BYTES) + static_cast<size_t>(ctas) * 128u * static_cast<size_t>(bn) * 4u;
}

template <int BN, typename OutT>
static int streamk_prepare() {
    int dev = 0;
    cudaGetDevice(&dev);
    static std::atomic<uint64_t> done{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return MICA_OK;
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_streamk_kernel<BN, OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GemmShape<BN, 4>::SMEM_BYTES);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    done.fetch_or(bit, std::memory_order_release);
    return MICA_OK;
}

template <int BN, typename OutT>
static int streamk_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& args,
                          int ctas, void* workspace, cudaStream_t stream) {
    int rc = streamk_prepare<BN, OutT>();
    if (rc) return rc;
    cudaError_t e = cudaMemsetAsync(workspace, 0, SK_FLAG_BYTES, stream);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    cfg.blockDim = dim3(GemmShape<BN, 4>::THREADS);
    cfg.dynamicSmemBytes = GemmShape<BN, 4>::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;     // every CTA resident: a FINISH waits on its neighbour
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, gemm_i8_streamk_kernel<BN, OutT>, ta, tb, tc, args,
                           static_cast<uint8_t*>(workspace));
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    return launch_status();
}

template <int BN>
static int streamk_dispatch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& g,
                            int c_dtype, int ctas, void* ws, cudaStream_t st) {
    if (c_dtype == MICA_DT_BF16) return streamk_launch<BN, __nv_bfloat16>(ta, tb, tc, g, ctas, ws, st);
    if (c_dtype == MICA_DT_FP16) return streamk_launch<BN, __half>(ta, tb, tc, g, ctas, ws, st);
    return streamk_launch<BN, float>(ta, tb, tc, g, ctas, ws, st);
}

// The GEMM's launch plan from its arguments (shared by the call and the workspace query).
struct GemmPlan {
    int bm, bn;
    bool streamk;
    int sk_ctas;
    size_t ws_bytes;
};

// Weight panel for multi-wave persistent grids (tile_origin): weights of more than kPanelBytes
// (N x K int8) are swept in near-equal panels of at most that size, each over all of M. Measured
// on the 49.8 MB gate_up weights at M = 32768, row-major order read them about eight times from
// DRAM; one 25 MB panel stays in L2 across the waves that use it, at the price of reading A once
// per panel.
constexpr size_t kPanelBytes = static_cast<size_t>(24) << 20;
static int gemm_panel(int N, int K, int bn) {
    const size_t wb = static_cast<size_t>(N) * static_cast<size_t>(K);
    if (wb <= kPanelBytes) return 0;
    const int num_n = (N + bn - 1) / bn;
    const int panels = static_cast<int>((wb + kPanelBytes - 1) / kPanelBytes);
    return (num_n + panels - 1) / panels;
}

static int gemm_tile_args_ok(int block_m, int block_n, int max_ctas, int splits) {
    if (block_m != 0 && block_m != 128 && block_m != 256) return MICA_ERR_ARG;
    if (block_n != 0 && block_n != 64 && block_n != 128 && block_n != 256 && block_n != 320) return MICA_ERR_ARG;
    if (block_m == 256 && (block_n == 64 || block_n == 320)) return MICA_ERR_ARG;
    if (block_n == 320 && (splits > 1 || splits == MICA_SPLIT_STREAM_K)) return MICA_ERR_ARG;
    if (max_ctas < 0 || splits < MICA_SPLIT_STREAM_K || splits > 8 || (splits > 1 && block_m == 256) ||
        (splits == MICA_SPLIT_STREAM_K && (block_m == 256 || max_ctas > 0)))
        return MICA_ERR_ARG;
    return MICA_OK;
}

static int gemm_plan(int M, int N, int K, int block_m, int block_n, int max_ctas, int splits, int sms,
                     GemmPlan* p) {
    if (int rc = gemm_tile_args_ok(block_m, block_n, max_ctas, splits)) return rc;
    int bm = block_m, bn = block_n;
    if (bm == 0 && bn == 0) {
        pick_tile(M, N, sms, &bm, &bn);
    } else if (bm == 0) {
        bm = 128;
    } else if (bn == 0) {
        int pm = 0;
        pick_tile(M, N, sms, &pm, &bn);
        if (bm == 256 && bn == 64) bn = 128;
        if (bm == 256 && bn == 320) bn = 256;
    }
    // 128 x 320 tiles need one CTA per tile and take no K split: a capped grid, a forced cluster
    // split or forced stream-K keeps the library's width choice at 256
    if (block_n == 0 && bn == 320 && (max_ctas > 0 || splits > 1 || splits == MICA_SPLIT_STREAM_K)) bn = 256;
    p->bm = bm;
    p->bn = bn;
    p->streamk = false;
    p->sk_ctas = 0;
    p->ws_bytes = 0;
    if (bm != 128 || max_ctas > 0) return MICA_OK;
    const long tiles = static_cast<long>((M + 127) / 128) * ((N + bn - 1) / bn);
    const int num_kb = (K + 127) / 128;
    if (splits == MICA_SPLIT_STREAM_K) {
        if ((bn != 128 && bn != 256) || sms > 256) return MICA_ERR_UNSUPPORTED;
        p->streamk = true;
    } else if (splits == 0 && (bn == 128 || bn == 256) && want_streamk(tiles, num_kb, sms)) {
        p->streamk = true;
    }
    if (p->streamk) {
        p->sk_ctas = static_cast<int>(tiles < sms ? tiles : sms);
        p->ws_bytes = streamk_ws_bytes(p->sk_ctas, bn);
    }
    return MICA_OK;
}

}  // namespace mica_host

using namespace mica_host;

// ======================================================================================
// entry points (C linkage comes from their declarations in include/mica_w8a8.h)
// ======================================================================================

const char* mica_last_cuda_error(void) { return t_err; }

int mica_query(int device, mica_caps* caps) {
    if (!caps) return MICA_ERR_ARG;
    memset(caps, 0, sizeof(*caps));
    caps->device = device;
    caps->abi_version = MICA_ABI_VERSION;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    if (device < 0 || device >= n) return MICA_ERR_ARG;
    if ((e = cudaDeviceGetAttribute(&caps->cc_major, cudaDevAttrComputeCapabilityMajor, device)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&caps->cc_minor, cudaDevAttrComputeCapabilityMinor, device)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&caps->sm_count, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&caps->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) !=
            cudaSuccess) {
        set_cuda_error(e);
        return MICA_ERR_CUDA;
    }
    caps->supported = (caps->cc_major == 10 && caps->cc_minor == 0 && caps->max_smem_optin >= 232448) ? 1 : 0;
    if (caps->supported) {
        int prev = 0;
        if ((e = cudaGetDevice(&prev)) != cudaSuccess || (e = cudaSetDevice(device)) != cudaSuccess) {
            set_cuda_error(e);
            return MICA_ERR_CUDA;
        }
        int rc = pair_prepare<256, __nv_bfloat16>(&caps->pair_clusters);
        cudaSetDevice(prev);
        if (rc) return rc;
    }
    return MICA_OK;
}

int mica_preload(int* n_kernels) {
    int rc = check_device(nullptr);
    if (rc) return rc;
    int n = 0;
#define PREP(BN, EPI, T)                                                            \
    if ((rc = gemm_prepare<BN, EPI, T, DequantWarps<BN>::EW>()) != MICA_OK) return rc; \
    ++n;
    PREP(64, EPI_DEQUANT, __nv_bfloat16)
    PREP(128, EPI_DEQUANT, __nv_bfloat16)
    PREP(256, EPI_DEQUANT, __nv_bfloat16)
    PREP(64, EPI_DEQUANT, __half)
    PREP(128, EPI_DEQUANT, __half)
    PREP(256, EPI_DEQUANT, __half)
    PREP(64, EPI_DEQUANT, float)
    PREP(128, EPI_DEQUANT, float)
    PREP(256, EPI_DEQUANT, float)
    PREP(320, EPI_DEQUANT, __nv_bfloat16)
    PREP(320, EPI_DEQUANT, __half)
    PREP(320, EPI_DEQUANT, float)
#undef PREP
    if ((rc = gemm_prepare<128, EPI_SWIGLU, __nv_bfloat16, 8>()) != MICA_OK) return rc;
    if ((rc = gemm_prepare<256, EPI_SWIGLU, __nv_bfloat16, 8>()) != MICA_OK) return rc;
    n += 2;
    int clusters = 0;
#define PREP_PAIR(BN, T)                                               \
    if ((rc = pair_prepare<BN, T>(&clusters)) != MICA_OK) return rc; \
    ++n;
    PREP_PAIR(128, __nv_bfloat16)
    PREP_PAIR(256, __nv_bfloat16)
    PREP_PAIR(128, __half)
    PREP_PAIR(256, __half)
    PREP_PAIR(128, float)
    PREP_PAIR(256, float)
#undef PREP_PAIR
    int dev = 0;
    cudaGetDevice(&dev);
    if ((rc = splitk_prepare_all<64>(dev)) || (rc = splitk_prepare_all<128>(dev)) ||
        (rc = splitk_prepare_all<256>(dev)))
        return rc;
    n += 9;
#define PREP_SK(BN, T)                                           \
    if ((rc = streamk_prepare<BN, T>()) != MICA_OK) return rc; \
    ++n;
    PREP_SK(128, __nv_bfloat16)
    PREP_SK(256, __nv_bfloat16)
    PREP_SK(128, __half)
    PREP_SK(256, __half)
    PREP_SK(128, float)
    PREP_SK(256, float)
#undef PREP_SK
    if (n_kernels) *n_kernels = n;
    return MICA_OK;
}

int mica_device_error(int* code, void* stream) {
    if (!code) return MICA_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    int v = 0;
    if ((e = cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int))) != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    const int zero = 0;
    if ((e = cudaMemcpyToSymbol(g_dev_error, &zero, sizeof(int))) != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    *code = v;
    return MICA_OK;
}

// ---------------------------------------------------------------------------------------
template <typename T>
static void norm_warp_launch(const QuantArgs& a, int nvec, cudaStream_t st) {
    const dim3 grid(static_cast<unsigned>((a.M + 3) / 4)), block(128);
    if (nvec <= 32 * 10) norm_rows_warp_kernel<T, 10><<<grid, block, 0, st>>>(a);
    else norm_rows_warp_kernel<T, 16><<<grid, block, 0, st>>>(a);
}

// Rows wider than this many 8-element vectors (K > 4096) take eight vectors per thread: on B200
// that took K = 9728 from 6.3 to 6.7 TB/s; K <= 4096 keeps four (5.8 vs 5.4 TB/s at K = 2560).
constexpr int PACKED_QV8_FROM = 512;
template <typename T>
static int packed_quant_launch(const QuantArgs& a, int nvec, cudaStream_t st) {
    const int qvp = nvec > PACKED_QV8_FROM ? 8 : 4;
    const int threads = ((nvec + qvp - 1) / qvp + 31) / 32 * 32;
    if (threads > 512) return MICA_ERR_UNSUPPORTED;
    if (qvp == 8) quant_rows_packed_kernel<T, 8><<<a.M, threads, 0, st>>>(a);
    else quant_rows_packed_kernel<T, 4><<<a.M, threads, 0, st>>>(a);
    return launch_status();
}

static int quant_launch(const QuantArgs& a, int dtype, int kind, cudaStream_t st) {
    const int nvec = a.K / 8;
    if (kind == QK_PLAIN && a.inv == nullptr && (dtype == MICA_DT_BF16 || dtype == MICA_DT_FP16) &&
        nvec <= 8 * 512) {
        return dtype == MICA_DT_BF16 ? packed_quant_launch<__nv_bfloat16>(a, nvec, st)
                                     : packed_quant_launch<__half>(a, nvec, st);
    }
    if (kind == QK_NORM && nvec <= 32 * 16 && (dtype == MICA_DT_BF16 || dtype == MICA_DT_FP16)) {
        // rows up to 4096 wide: one warp per row (no block barriers)
        if (dtype == MICA_DT_BF16) norm_warp_launch<__nv_bfloat16>(a, nvec, st);
        else norm_warp_launch<__half>(a, nvec, st);
        return launch_status();
    }
    int threads = ((nvec + QV - 1) / QV + 31) / 32 * 32;
    if (threads < 32) threads = 32;
    if (threads > 1024) return MICA_ERR_UNSUPPORTED;
    const dim3 grid(a.M), block(threads);
    if (kind != QK_PLAIN && dtype == MICA_DT_FP32) return MICA_ERR_ARG;
#define QLAUNCH_T(T, MAXT)                                                                    \
    if (kind == QK_NORM) quant_rows_kernel<T, QK_NORM, MAXT><<<grid, block, 0, st>>>(a);      \
    else if (kind == QK_SWIGLU) quant_rows_kernel<T, QK_SWIGLU, MAXT><<<grid, block, 0, st>>>(a); \
    else quant_rows_kernel<T, QK_PLAIN, MAXT><<<grid, block, 0, st>>>(a);
#define QLAUNCH(MAXT)                                                                         \
    if (dtype == MICA_DT_BF16) {                                                              \
        QLAUNCH_T(__nv_bfloat16, MAXT)                                                        \
    } else if (dtype == MICA_DT_FP16) {                                                       \
        QLAUNCH_T(__half, MAXT)                                                               \
    } else {                                                                                  \
        quant_rows_kernel<float, QK_PLAIN, MAXT><<<grid, block, 0, st>>>(a);                  \
    }
    if (threads <= 512) {
        QLAUNCH(512)
    } else {
        QLAUNCH(1024)
    }
#undef QLAUNCH
#undef QLAUNCH_T
    return launch_status();
}

int mica_act_quant(const void* x, int x_dtype, long ldx, const float* inv, int8_t* q, long ldq, float* s, int M,
                   int K, int round_mode, void* stream) {
    if (!x || !q || !s || x_dtype < 0 || x_dtype > 2 || (round_mode != 0 && round_mode != 1)) return MICA_ERR_ARG;
    if (M < 0 || K < 8 || (K & 7) || ldx < K || ldq < K) return MICA_ERR_SHAPE;
    if (static_cast<long>(M) * (ldx > ldq ? ldx : ldq) >= (1L << 40)) return MICA_ERR_RANGE;
    const size_t es = dt_size(x_dtype);
    if (!aligned16(x) || !aligned16(q) || (inv && !aligned16(inv)) || (ldx * es) % 16 || ldq % 16) return MICA_ERR_ALIGN;
    int rc = check_device(nullptr);
    if (rc) return rc;
    if (M == 0) return MICA_OK;
    QuantArgs a = {};
    a.x = x; a.ldx = ldx; a.inv = inv; a.q = q; a.ldq = ldq; a.s = s;
    a.M = M; a.K = K; a.round_mode = round_mode;
    return quant_launch(a, x_dtype, QK_PLAIN, static_cast<cudaStream_t>(stream));
}

int mica_rmsnorm_quant(const void* x, int x_dtype, long ldx, const void* residual, long ldr, const void* gamma,
                       int norm_style, float eps, const float* inv, void* y_out, long ldy, void* sum_out, long ldsum,
                       int8_t* q, long ldq, float* s, int M, int K, int round_mode, void* stream) {
    if (!x || !gamma || (!q != !s) || (!q && !y_out) || (x_dtype != MICA_DT_BF16 && x_dtype != MICA_DT_FP16) ||
        (round_mode != 0 && round_mode != 1) || (norm_style != MICA_NORM_OFFSET && norm_style != MICA_NORM_WEIGHT))
        return MICA_ERR_ARG;
    if (M < 0 || K < 8 || (K & 7) || ldx < K || (q && ldq < K) || (residual && ldr < K) || (y_out && ldy < K) ||
        (sum_out && ldsum < K))
        return MICA_ERR_SHAPE;
    if (sum_out && !residual) return MICA_ERR_ARG;
    const long es = 2;
    if (!aligned16(x) || !aligned16(gamma) || (q && !aligned16(q)) || (inv && !aligned16(inv)) ||
        (residual && (!aligned16(residual) || (ldr * es) % 16)) || (y_out && (!aligned16(y_out) || (ldy * es) % 16)) ||
        (sum_out && (!aligned16(sum_out) || (ldsum * es) % 16)) || (ldx * es) % 16 || ldq % 16)
        return MICA_ERR_ALIGN;
    int rc = check_device(nullptr);
    if (rc) return rc;
    if (M == 0) return MICA_OK;
    QuantArgs a = {};
    a.x = x; a.ldx = ldx; a.residual = residual; a.ldr = ldr; a.gamma = gamma; a.norm_style = norm_style;
    a.eps = eps; a.inv = inv; a.y_out = y_out; a.ldy = ldy; a.sum_out = sum_out; a.ldsum = ldsum;
    a.q = q; a.ldq = ldq; a.s = s; a.M = M; a.K = K; a.round_mode = round_mode;
    return quant_launch(a, x_dtype, QK_NORM, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------
static int gemm_checks(const int8_t* A, long lda, const int8_t* B, long ldb, const float* sa, const float* sb,
                       const float* bias, const void* C, int c_dtype, long ldc, int M, int N, int K) {
    if (!A || !B || !sa || !sb || !C || c_dtype < 0 || c_dtype > 2) return MICA_ERR_ARG;
    if (M < 0 || N < 1 || K < 16 || (K & 15) || lda < K || ldb < K || ldc < N) return MICA_ERR_SHAPE;
    if (M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return MICA_ERR_RANGE;
    const long es = static_cast<long>(dt_size(c_dtype));
    if (!aligned16(A) || !aligned16(B) || !aligned16(C) || lda % 16 || ldb % 16 || (ldc * es) % 16)
        return MICA_ERR_ALIGN;
    (void)sa; (void)sb; (void)bias;
    return MICA_OK;
}

template <int BN>
static int gemm_dispatch_out(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& g,
                             int c_dtype, int grid, cudaStream_t st) {
    constexpr int EW = DequantWarps<BN>::EW;
    if (c_dtype == MICA_DT_BF16) return gemm_launch<BN, EPI_DEQUANT, __nv_bfloat16, EW>(ta, tb, tc, g, grid, false, st);
    if (c_dtype == MICA_DT_FP16) return gemm_launch<BN, EPI_DEQUANT, __half, EW>(ta, tb, tc, g, grid, false, st);
    return gemm_launch<BN, EPI_DEQUANT, float, EW>(ta, tb, tc, g, grid, false, st);
}

size_t mica_w8a8_gemm_workspace_bytes(int M, int N, int K, int block_m, int block_n, int max_ctas, int splits) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    int sms = 0;
    if (check_device(&sms)) return 0;
    GemmPlan p;
    if (gemm_plan(M, N, K, block_m, block_n, max_ctas, splits, sms, &p)) return 0;
    return p.ws_bytes;
}

int mica_w8a8_gemm_cfg(const int8_t* A, long lda, const int8_t* B, long ldb, const float* sa, const float* sb,
                       const float* bias, void* C, int c_dtype, long ldc, int M, int N, int K, int block_m,
                       int block_n, int max_ctas, int splits, void* stream) {
    return mica_w8a8_gemm_ex(A, lda, B, ldb, sa, sb, bias, C, c_dtype, ldc, M, N, K, block_m, block_n, max_ctas,
                             splits, nullptr, 0, stream);
}

int mica_w8a8_gemm_ex(const int8_t* A, long lda, const int8_t* B, long ldb, const float* sa, const float* sb,
                      const float* bias, void* C, int c_dtype, long ldc, int M, int N, int K, int block_m,
                      int block_n, int max_ctas, int splits, void* workspace, size_t workspace_bytes,
                      void* stream) {
    int rc = gemm_checks(A, lda, B, ldb, sa, sb, bias, C, c_dtype, ldc, M, N, K);
    if (rc) return rc;
    if ((rc = gemm_tile_args_ok(block_m, block_n, max_ctas, splits))) return rc;
    if (workspace && !aligned16(workspace)) return MICA_ERR_ALIGN;
    int sms = 0;
    if ((rc = check_device(&sms))) return rc;
    GemmPlan plan;
    if ((rc = gemm_plan(M, N, K, block_m, block_n, max_ctas, splits, sms, &plan))) return rc;
    if (plan.streamk) {
        const bool forced = splits == MICA_SPLIT_STREAM_K;
        if (!workspace || workspace_bytes < plan.ws_bytes) {
            if (forced) return MICA_ERR_WORKSPACE;
            plan.streamk = false;                 // library choice without room for it: data-parallel
        }
    }
    if (M == 0) return MICA_OK;
    const int bm = plan.bm, bn = plan.bn;
    CUtensorMap ta, tb, tc;
    const CUtensorMapDataType cdt = c_dtype == MICA_DT_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                    : c_dtype == MICA_DT_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const uint32_t es = static_cast<uint32_t>(dt_size(c_dtype));
    // A CTA of a pair loads 128 rows of A and bn/2 rows of B; a 320-wide tile loads its B rows
    // as two 160-row boxes.
    const uint32_t b_box = (bm == 256 || bn == 320) ? static_cast<uint32_t>(bn / 2) : static_cast<uint32_t>(bn);
    if ((rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, lda, 128, 128)) ||
        (rc = make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldb, 128, b_box)) ||
        (rc = make_tmap_2d(&tc, C, cdt, N, M, ldc * es, 128 / es, 32)))
        return rc;
    GemmArgs g = {};
    g.sa = sa; g.sb = sb; g.bias = bias; g.M = M; g.N = N; g.K = K;
    g.panel = gemm_panel(N, K, bn);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (bm == 256) {
        const long tiles = static_cast<long>((M + 255) / 256) * ((N + bn - 1) / bn);
        if (bn == 256) {
            if (c_dtype == MICA_DT_BF16) return pair_launch<256, __nv_bfloat16>(ta, tb, tc, g, tiles, max_ctas, st);
            if (c_dtype == MICA_DT_FP16) return pair_launch<256, __half>(ta, tb, tc, g, tiles, max_ctas, st);
            return pair_launch<256, float>(ta, tb, tc, g, tiles, max_ctas, st);
        }
        if (c_dtype == MICA_DT_BF16) return pair_launch<128, __nv_bfloat16>(ta, tb, tc, g, tiles, max_ctas, st);
        if (c_dtype == MICA_DT_FP16) return pair_launch<128, __half>(ta, tb, tc, g, tiles, max_ctas, st);
        return pair_launch<128, float>(ta, tb, tc, g, tiles, max_ctas, st);
    }
    if (plan.streamk) {
        if (bn == 256) return streamk_dispatch<256>(ta, tb, tc, g, c_dtype, plan.sk_ctas, workspace, st);
        return streamk_dispatch<128>(ta, tb, tc, g, c_dtype, plan.sk_ctas, workspace, st);
    }
    const long tiles = static_cast<long>((M + 127) / 128) * ((N + bn - 1) / bn);
    if (bn == 320) {
        // one accumulator buffer per CTA: one tile per CTA, all in one wave
        if (tiles > sms || (max_ctas > 0 && tiles > max_ctas)) return MICA_ERR_UNSUPPORTED;
        return gemm_dispatch_out<320>(ta, tb, tc, g, c_dtype, static_cast<int>(tiles), st);
    }
    if (splits != 1 && max_ctas == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if ((rc = bn == 256 ? splitk_prepare_all<256>(dev) : bn == 128 ? splitk_prepare_all<128>(dev)
                                                                        : splitk_prepare_all<64>(dev)))
            return rc;
        const int num_kb = (K + 127) / 128;
        int s = splits;
        if (s == 0) {
            s = choose_splits(dev, bn, tiles, num_kb, sms);
        } else {
            const int per = (num_kb + s - 1) / s;
            const int co = g_splitk_clusters[dev][bn_index(bn)][s].load();
            if ((s - 1) * per >= num_kb || co <= 0) return MICA_ERR_UNSUPPORTED;   // a rank would be empty
        }
        if (s > 1) {
            if (bn == 256) return splitk_dispatch<256>(ta, tb, tc, g, c_dtype, tiles, s, st);
            if (bn == 128) return splitk_dispatch<128>(ta, tb, tc, g, c_dtype, tiles, s, st);
            return splitk_dispatch<64>(ta, tb, tc, g, c_dtype, tiles, s, st);
        }
    }
    int grid = static_cast<int>(tiles < sms ? tiles : sms);
    if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
    if (bn == 256) return gemm_dispatch_out<256>(ta, tb, tc, g, c_dtype, grid, st);
    if (bn == 128) return gemm_dispatch_out<128>(ta, tb, tc, g, c_dtype, grid, st);
    return gemm_dispatch_out<64>(ta, tb, tc, g, c_dtype, grid, st);
}

int mica_w8a8_gemm(const int8_t* A, long lda, const int8_t* B, long ldb, const float* sa, const float* sb,
                   const float* bias, void* C, int c_dtype, long ldc, int M, int N, int K, void* stream) {
    return mica_w8a8_gemm_cfg(A, lda, B, ldb, sa, sb, bias, C, c_dtype, ldc, M, N, K, 0, 0, 0, 0, stream);
}

// ---------------------------------------------------------------------------------------
// workspace layout: [row_amax: M uint32, padded to 16 B][grid counter: 16 B]
size_t mica_swiglu_workspace_bytes(int M) {
    if (M < 0) return 0;
    return (static_cast<size_t>(M) * 4 + 15) / 16 * 16 + 16;
}

// Argument checks shared by the two fused SwiGLU entry points (no CUDA call is made).
static int swiglu_args_ok(const int8_t* A, long lda, const int8_t* Bgu, long ldb, const float* sa, const float* sgu,
                          const float* inv_h, const void* h_out, long ldh, const int8_t* q_out, long ldq,
                          const float* s_out, int M, int I, int K, int round_mode) {
    if (!A || !Bgu || !sa || !sgu || !h_out || !q_out || !s_out || (round_mode != 0 && round_mode != 1))
        return MICA_ERR_ARG;
    if (M < 0 || I < 16 || (I & 15) || K < 16 || (K & 15) || lda < K || ldb < K || ldh < I || ldq < I)
        return MICA_ERR_SHAPE;
    if (M > (1 << 30) || I > (1 << 29) || K > (1 << 30)) return MICA_ERR_RANGE;
    if (!aligned16(A) || !aligned16(Bgu) || !aligned16(h_out) || !aligned16(q_out) || lda % 16 || ldb % 16 ||
        (ldh * 2) % 16 || ldq % 16 || (inv_h && !aligned16(inv_h)))
        return MICA_ERR_ALIGN;
    return MICA_OK;
}

int mica_w8a8_gemm_swiglu_quant(const int8_t* A, long lda, const int8_t* Bgu, long ldb, const float* sa,
                                const float* sgu, const float* bias_gu, const float* inv_h, void* h_out, long ldh,
                                int8_t* q_out, long ldq, float* s_out, int M, int I, int K, int round_mode,
                                void* workspace, size_t workspace_bytes, void* stream) {
    if (int arc = swiglu_args_ok(A, lda, Bgu, ldb, sa, sgu, inv_h, h_out, ldh, q_out, ldq, s_out, M, I, K, round_mode))
        return arc;
    if (!workspace || !aligned16(workspace)) return workspace ? MICA_ERR_ALIGN : MICA_ERR_ARG;
    if (workspace_bytes < mica_swiglu_workspace_bytes(M)) return MICA_ERR_WORKSPACE;
    int sms = 0;
    int rc = check_device(&sms);
    if (rc) return rc;
    if (M == 0) return MICA_OK;
    const int N = 2 * I;
    const long tiles256 = static_cast<long>((M + 127) / 128) * ((N + 255) / 256);
    const int bn = tiles256 >= sms ? 256 : 128;
    CUtensorMap ta, tb, th;
    if ((rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, lda, 128, 128)) ||
        (rc = make_tmap_2d(&tb, Bgu, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldb, 128, bn)) ||
        (rc = make_tmap_2d(&th, h_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, I, M, ldh * 2, 64, 32)))
        return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned* amax = static_cast<unsigned*>(workspace);
    unsigned* sync = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + (static_cast<size_t>(M) * 4 + 15) / 16 * 16);
    cudaError_t e = cudaMemsetAsync(workspace, 0, mica_swiglu_workspace_bytes(M), st);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    GemmArgs g = {};
    g.sa = sa; g.sb = sgu; g.bias = bias_gu; g.M = M; g.N = N; g.K = K; g.round_mode = round_mode;
    g.row_amax = amax; g.grid_sync = sync;
    g.h = static_cast<const __nv_bfloat16*>(h_out); g.ldh = ldh; g.q_out = q_out; g.ldq = ldq; g.s_out = s_out;
    g.inv_h = inv_h;
    g.panel = gemm_panel(N, K, bn);
    const long tiles = static_cast<long>((M + 127) / 128) * ((N + bn - 1) / bn);
    const int grid = static_cast<int>(tiles < sms ? tiles : sms);
    if (bn == 256) return gemm_launch<256, EPI_SWIGLU, __nv_bfloat16, 8>(ta, tb, th, g, grid, true, st);
    return gemm_launch<128, EPI_SWIGLU, __nv_bfloat16, 8>(ta, tb, th, g, grid, true, st);
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant of the fused SwiGLU chain, for callers that cannot call
// cudaMalloc (see include/mica_w8a8.h). Its scratch -- one row-max word per token plus the
// grid-barrier counter, laid out exactly as the workspace of mica_w8a8_gemm_swiglu_quant --
// is this file-scope device array. Each GPU that loads the library holds one copy until
// the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MICA_NOALLOC_SCRATCH_BYTES];
static_assert(MICA_NOALLOC_SCRATCH_BYTES >= (static_cast<size_t>(MICA_NOALLOC_MAX_ROWS) * 4 + 15) / 16 * 16 + 16,
              "scratch must hold the workspace of MICA_NOALLOC_MAX_ROWS rows");

// Device address of g_noalloc_scratch per device. In host code the array's name is only a
// host-side stand-in, so the address is looked up once per device (with that device
// current) and cached; the lookup itself allocates nothing.
static void* g_noalloc_addr[kMaxDev] = {};
static std::mutex g_noalloc_lock;

static int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
    if (dev < 0 || dev >= kMaxDev) return MICA_ERR_ARCH;
    std::lock_guard<std::mutex> g(g_noalloc_lock);
    if (g_noalloc_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            set_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
            return MICA_ERR_CUDA;
        }
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return MICA_OK;
}

int mica_w8a8_gemm_swiglu_quant_noalloc(const int8_t* A, long lda, const int8_t* Bgu, long ldb, const float* sa,
                                        const float* sgu, const float* bias_gu, const float* inv_h, void* h_out,
                                        long ldh, int8_t* q_out, long ldq, float* s_out, int M, int I, int K,
                                        int round_mode, void* stream) {
    // the same argument checks as the workspace entry point, before any CUDA call
    int rc = swiglu_args_ok(A, lda, Bgu, ldb, sa, sgu, inv_h, h_out, ldh, q_out, ldq, s_out, M, I, K, round_mode);
    if (rc) return rc;
    if (M > MICA_NOALLOC_MAX_ROWS) return MICA_ERR_WORKSPACE;   // beyond the fixed scratch: refuse up front
    rc = check_device(nullptr);
    if (rc) return rc;
    void* scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    // The shared entry point clears the rows it uses (cudaMemsetAsync, no allocation)
    // before launching, so stale contents from the previous call do not leak in.
    return mica_w8a8_gemm_swiglu_quant(A, lda, Bgu, ldb, sa, sgu, bias_gu, inv_h, h_out, ldh, q_out, ldq, s_out, M,
                                       I, K, round_mode, scratch, MICA_NOALLOC_SCRATCH_BYTES, stream);
}

// ---------------------------------------------------------------------------------------
int mica_swiglu_quant(const void* g, long ldg, const void* u, long ldu, int dtype, const float* inv, void* h_out,
                      long ldh, int8_t* q, long ldq, float* s, int M, int I, int round_mode, void* stream) {
    if (!g || !u || (!q != !s) || (!q && !h_out) || (dtype != MICA_DT_BF16 && dtype != MICA_DT_FP16) ||
        (round_mode != 0 && round_mode != 1))
        return MICA_ERR_ARG;
    if (M < 0 || I < 8 || (I & 7) || ldg < I || ldu < I || (h_out && ldh < I) || (q && ldq < I))
        return MICA_ERR_SHAPE;
    const long ld_max = std::max(std::max(ldg, ldu), std::max(h_out ? ldh : 0L, q ? ldq : 0L));
    if (static_cast<long>(M) * ld_max >= (1L << 40)) return MICA_ERR_RANGE;
    if (!aligned16(g) || !aligned16(u) || (h_out && !aligned16(h_out)) || (q && !aligned16(q)) ||
        (inv && !aligned16(inv)) || (ldg * 2) % 16 || (ldu * 2) % 16 || (h_out && (ldh * 2) % 16) ||
        (q && ldq % 16))
        return MICA_ERR_ALIGN;
    int rc = check_device(nullptr);
    if (rc) return rc;
    if (M == 0) return MICA_OK;
    QuantArgs a = {};
    a.x = g; a.ldx = ldg; a.residual = u; a.ldr = ldu; a.inv = inv; a.y_out = h_out; a.ldy = ldh;
    a.q = q; a.ldq = ldq; a.s = s; a.M = M; a.K = I; a.round_mode = round_mode;
    return quant_launch(a, dtype, QK_SWIGLU, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------
int mica_option_logits(const void* h, int h_dtype, long ldh, const void* gamma, int norm_style, float eps,
                       const float* rows, int n_rows, int D, const int* lo, const int* hi, float* logits, float* probs,
                       int B, void* stream) {
    if (!h || !rows || !logits || h_dtype < 0 || h_dtype > 2 ||
        (norm_style != MICA_NORM_OFFSET && norm_style != MICA_NORM_WEIGHT))
        return MICA_ERR_ARG;
    if (gamma && h_dtype == MICA_DT_FP32) return MICA_ERR_UNSUPPORTED;
    if (B < 0 || n_rows < 1 || n_rows > 4096 || D < 8 || (D & 7) || D > 4096 || ldh < D) return MICA_ERR_SHAPE;
    const long es = static_cast<long>(dt_size(h_dtype));
    if (!aligned16(h) || !aligned16(rows) || (gamma && !aligned16(gamma)) || (ldh * es) % 16) return MICA_ERR_ALIGN;
    int rc = check_device(nullptr);
    if (rc) return rc;
    if (B == 0) return MICA_OK;
    ReadoutArgs a = {};
    a.h = h; a.ldh = ldh; a.gamma = gamma; a.norm_style = norm_style; a.eps = eps; a.rows = rows;
    a.n_rows = n_rows; a.D = D; a.lo = lo; a.hi = hi; a.logits = logits; a.probs = probs; a.B = B;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid((n_rows + RO_WARPS - 1) / RO_WARPS), block(RO_WARPS * 32);
    const size_t smem = static_cast<size_t>(D) * sizeof(float);
#define RO_LAUNCH(T)                                                                                   \
    do {                                                                                               \
        if (D <= 1024) option_logits_kernel<T, 8><<<grid, block, smem, st>>>(a);                       \
        else if (D <= 2048) option_logits_kernel<T, 16><<<grid, block, smem, st>>>(a);                 \
        else if (D <= 2560) option_logits_kernel<T, 20><<<grid, block, smem, st>>>(a);                 \
        else option_logits_kernel<T, 32><<<grid, block, smem, st>>>(a);                                \
    } while (0)
    if (h_dtype == MICA_DT_BF16) RO_LAUNCH(__nv_bfloat16);
    else if (h_dtype == MICA_DT_FP16) RO_LAUNCH(__half);
    else RO_LAUNCH(float);
#undef RO_LAUNCH
    if ((rc = launch_status())) return rc;
    if (probs) {
        option_softmax_kernel<<<(B + 7) / 8, 256, 0, st>>>(a);
        return launch_status();
    }
    return MICA_OK;
}

// ---------------------------------------------------------------------------------------
int mica_qk_norm_rope(void* qkv, long ld, const void* q_w, const void* k_w, const void* cos, const void* sin,
                      const int64_t* pos, long pos0, int S, int H, int KV, int D, float eps, void* stream) {
    if (!qkv || !cos || !sin || (H > 0 && !q_w) || (KV > 0 && !k_w)) return MICA_ERR_ARG;
    if (S < 0 || H < 0 || KV < 0 || (D != 64 && D != 128) || ld < static_cast<long>(H + KV) * D || pos0 < 0)
        return MICA_ERR_SHAPE;
    const auto al8 = [](const void* ptr) { return ptr == nullptr || reinterpret_cast<uintptr_t>(ptr) % 8 == 0; };
    if (!aligned16(qkv) || (ld * 2) % 16 || !al8(cos) || !al8(sin) || !al8(q_w) || !al8(k_w)) return MICA_ERR_ALIGN;
    int rc = check_device(nullptr);
    if (rc) return rc;
    const long warps = static_cast<long>(S) * (H + KV);
    if (warps == 0) return MICA_OK;
    if (warps > (1L << 31) * 8 / 256 * 32) return MICA_ERR_RANGE;
    QkRopeArgs a = {};
    a.qkv = static_cast<__nv_bfloat16*>(qkv); a.ld = ld;
    a.q_w = static_cast<const __nv_bfloat16*>(q_w); a.k_w = static_cast<const __nv_bfloat16*>(k_w);
    a.cos = static_cast<const __nv_bfloat16*>(cos); a.sin = static_cast<const __nv_bfloat16*>(sin);
    a.pos = reinterpret_cast<const long*>(pos); a.pos0 = pos0; a.S = S; a.H = H; a.KV = KV; a.eps = eps;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (D == 128) {
        // one warp per token (cos/sin and weights held across the token's heads)
        const unsigned blocks = static_cast<unsigned>((static_cast<long>(S) * 32 + 255) / 256);
        qk_norm_rope_token_kernel<<<blocks, 256, 0, st>>>(a);
    } else {
        const unsigned blocks = static_cast<unsigned>((warps * 32 + 255) / 256);
        qk_norm_rope_kernel<64><<<blocks, 256, 0, st>>>(a);
    }
    return launch_status();
}

// ---------------------------------------------------------------------------------------
int mica_attention_prefill(const void* qkv, long ld_qkv, void* out, long ld_out, int B, int L, int H, int KV, int D,
                           float scale, void* stream) {
    if (!qkv || !out || !(scale > 0.f)) return MICA_ERR_ARG;
    if (B < 0 || L < 0 || H < 1 || KV < 1 || H % KV || D != ATT_D || ld_qkv < static_cast<long>(H + 2 * KV) * D ||
        ld_out < static_cast<long>(H) * D)
        return MICA_ERR_SHAPE;
    if (!aligned16(qkv) || !aligned16(out) || (ld_qkv * 2) % 16 || (ld_out * 2) % 16) return MICA_ERR_ALIGN;
    const long rows = static_cast<long>(B) * L;
    const long ctas = static_cast<long>(B) * ((L + 2 * ATT_BM - 1) / (2 * ATT_BM)) * H;
    if (rows > (1L << 31) - 1 || ctas > (1L << 31) - 1) return MICA_ERR_RANGE;
    int rc = check_device(nullptr);
    if (rc) return rc;
    if (rows == 0) return MICA_OK;
    {
        int dev = 0;
        cudaGetDevice(&dev);
        static std::atomic<uint64_t> done{0};
        const uint64_t bit = 1ull << (dev & 63);
        if (!(done.load(std::memory_order_acquire) & bit)) {
            cudaError_t e = cudaFuncSetAttribute(attention_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 ATT_SMEM_BYTES);
            if (e != cudaSuccess) { set_cuda_error(e); return MICA_ERR_CUDA; }
            done.fetch_or(bit, std::memory_order_release);
        }
    }
    CUtensorMap tm;
    if ((rc = make_tmap_2d(&tm, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<uint64_t>(H + 2 * KV) * D,
                           static_cast<uint64_t>(rows), static_cast<uint64_t>(ld_qkv) * 2, 64, ATT_BM)))
        return rc;
    AttnArgs a = {};
    a.qkv = static_cast<const __nv_bfloat16*>(qkv); a.ld_qkv = ld_qkv;
    a.out = static_cast<__nv_bfloat16*>(out); a.ld_out = ld_out;
    a.B = B; a.L = L; a.H = H; a.KV = KV;
    a.scale_log2 = scale * 1.4426950408889634f;
    attention_fwd_kernel<<<static_cast<unsigned>(ctas), ATT_THREADS, ATT_SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(
        tm, a);
    return launch_status();
}

// ---------------------------------------------------------------------------------------
// Failure-detection self-test: one block waits on an mbarrier that never completes.
__global__ void selftest_wait_kernel(int* status, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    __shared__ uint32_t abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool ok = mbar_wait(&bar, 0, &abort_flag, MICA_DEV_TIMEOUT_SELFTEST, limit_ns);
        *status = ok ? MICA_DEV_OK : MICA_DEV_TIMEOUT_SELFTEST;
    }
}

int mica_selftest_wait_timeout(int* status_dev, int limit_us, void* stream) {
    if (!status_dev || limit_us < 1 || limit_us > 2000000) return MICA_ERR_ARG;
    int rc = check_device(nullptr);
    if (rc) return rc;
    selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        status_dev, static_cast<unsigned long long>(limit_us) * 1000ull);
    return launch_status();
}
