// C ABI of the ETHOS expert layer (declared in include/ethos_b200.h).
//
// Host-side orchestration only: argument checks, workspace partitioning,
// TMA tensor-map encoding and kernel launches on the caller's stream.  No
// device memory is allocated here.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <mutex>
#include <utility>

#include "ethos_b200.h"
#include "expert.cuh"
#include "expert_table.cuh"
#include "backward.cuh"
#include "gemm.cuh"
#include "gemm2sm.cuh"
#include "router.cuh"
#include "optim.cuh"
#include "fp32.cuh"

using namespace ethos;

// Scratch of ethos_router_forward_noalloc: the only device memory that entry
// point uses besides the caller's inputs and outputs.  In host code this name
// is a host-side stand-in, not a device address; noalloc_scratch() resolves
// the device address once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[ETHOS_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kAbiVersion = 6;

// The device GELU variants the kernels use, evaluated on x [n] (n even) into
// out [5, n]: gelu_erf, gelu_erf2 (pairs), gelu_erf_and_grad2 (value, then
// derivative) and gelu_erf_grad (ethos_test_gelu).
__global__ void k_test_gelu(const float* __restrict__ x, float* __restrict__ out, int64_t n) {
  const int64_t pairs = n / 2;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < pairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float2 v = reinterpret_cast<const float2*>(x)[i];
    float a0, a1, g0, g1, d0, d1;
    gelu_erf2(v.x, v.y, a0, a1);
    gelu_erf_and_grad2(v.x, v.y, g0, g1, d0, d1);
    reinterpret_cast<float2*>(out)[i] = make_float2(gelu_erf(v.x), gelu_erf(v.y));
    reinterpret_cast<float2*>(out + n)[i] = make_float2(a0, a1);
    reinterpret_cast<float2*>(out + 2 * n)[i] = make_float2(g0, g1);
    reinterpret_cast<float2*>(out + 3 * n)[i] = make_float2(d0, d1);
    reinterpret_cast<float2*>(out + 4 * n)[i] = make_float2(gelu_erf_grad(v.x), gelu_erf_grad(v.y));
  }
}

// Kernels this library has launched in this process (ethos_launch_count).
std::atomic<unsigned long long> g_launch_count{0};
inline void count_launch() { g_launch_count.fetch_add(1, std::memory_order_relaxed); }

// ------------------------------------------------------------ device cache --
struct DeviceInfo {
  int sm_count = 0;
  int major = 0;
  bool attrs_set = false;
};
std::mutex g_mu;
DeviceInfo g_dev[64];

int device_info(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ETHOS_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.sm_count == 0) {
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return ETHOS_ERR_CUDA;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return ETHOS_ERR_CUDA;
    d.sm_count = sms;
    d.major = major;
  }
  if (d.major != 10) return ETHOS_ERR_NO_DEVICE;
  if (!d.attrs_set) {
    bool ok = true;
    ok &= cudaFuncSetAttribute(k_score_topk<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, ROUTER_SMEM_BYTES) ==
          cudaSuccess;
    ok &= cudaFuncSetAttribute(k_score_topk<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, ROUTER_SMEM_BYTES) ==
          cudaSuccess;
    ok &= cudaFuncSetAttribute(k_score_topk<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, ROUTER_SMEM_BYTES) ==
          cudaSuccess;
    ok &= cudaFuncSetAttribute(k_expert_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, EX_SMEM_BYTES) ==
          cudaSuccess;
    ok &= cudaFuncSetAttribute(k_expert_gather, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               GATHER_SMEM_BYTES) == cudaSuccess;
    if (!ok) return ETHOS_ERR_CUDA;
    d.attrs_set = true;
  }
  *out = &d;
  return ETHOS_OK;
}

// Sets the dynamic shared-memory limit of a kernel once per device.
int smem_attr_once(const void* fn, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ETHOS_ERR_NO_DEVICE;
  static std::mutex mu;
  static const void* seen[64][32];
  static int nseen[64];
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < nseen[dev]; ++i)
    if (seen[dev][i] == fn) return ETHOS_OK;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return ETHOS_ERR_CUDA;
  if (nseen[dev] < 32) seen[dev][nseen[dev]++] = fn;
  return ETHOS_OK;
}

// ------------------------------------------------------------- tensor maps --
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Row-major bf16 matrix [rows, cols] (row pitch ld >= cols elements) read in
// boxes of 64 columns x box_rows rows with the 128-byte swizzle that the UMMA
// descriptors expect.
// box_cols 64, 32 or 16 (rows of 128, 64 or 32 bytes, with the swizzle of
// that width); the UMMA descriptor of the consuming kernel must match it.
int make_tmap_bf16(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int box_rows, int64_t ld = 0,
                   int box_cols = 64, CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return ETHOS_ERR_TENSOR_MAP;
  if (ld == 0) ld = cols;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0 || (ld * 2) % 16 != 0) return ETHOS_ERR_ALIGNMENT;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  if (box_cols != 64 && box_cols != 32 && box_cols != 16) return ETHOS_ERR_TENSOR_MAP;
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : (box_cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ETHOS_OK : ETHOS_ERR_TENSOR_MAP;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Optional per-stage timing: records stage_events[i] (a cudaEvent_t) on the
// stream at stage boundary i when the caller passed an array.
void mark(void* const* ev, int i, cudaStream_t s) {
  if (ev != nullptr && ev[i] != nullptr) cudaEventRecord(static_cast<cudaEvent_t>(ev[i]), s);
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ETHOS_OK : ETHOS_ERR_CUDA;
}

// Launch with programmatic stream serialization: the kernel may start while
// the previous kernel of the stream finishes (its set-up overlaps that tail)
// and waits in pdl_wait() for it before touching global memory.  Only kernels
// that call pdl_wait() before their first global access are launched so.
template <class... KArgs, class... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  if (cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) != cudaSuccess) return ETHOS_ERR_CUDA;
  return launch_status();
}

// Operand of a GEMM: bf16 matrix stored row-major with row pitch ld; K-major
// means stored [rows = M or N][K], MN-major means stored [K][M or N].
struct GemmOperand {
  const void* ptr;
  int64_t ld;
  bool mn_major;
};

int operand_tmap(CUtensorMap* m, const GemmOperand& o, int64_t mn, int64_t k, int mn_box) {
  if (o.mn_major) return make_tmap_bf16(m, o.ptr, k, mn, 64, o.ld);
  return make_tmap_bf16(m, o.ptr, mn, k, mn_box, o.ld);
}

// Launches D = A B^T on the generic kernel.  ksplit > 1 requires an epilogue
// that accumulates (EpiAtomicF32).  BN = 256 when N allows, else 128.
// tc: the output's tensor map, for an epilogue that stores through TMA
// (Epi::kTmaStore); other epilogues ignore the argument.
template <class Epi, bool AMN, bool BMN, int BN>
int launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, int ksplit, const Epi& epi,
                  int* err, cudaStream_t stream, const DeviceInfo& dev, int hold_unit = -1,
                  const CUtensorMap* tc = nullptr, const CUtensorMap* td = nullptr) {
  if (Epi::kTmaStore && tc == nullptr) return ETHOS_ERR_INVALID_ARG;
  if (GemmCfg<Epi>::kTmaOutputs == 2 && td == nullptr) return ETHOS_ERR_INVALID_ARG;
  auto kern = k_gemm<Epi, AMN, BMN, BN>;
  int st = smem_attr_once(reinterpret_cast<const void*>(kern), GemmCfg<Epi>::kSmem);
  if (st != ETHOS_OK) return st;
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * (N / BN);
  const int units = tiles * ksplit;
  const int grid = units < dev.sm_count ? units : dev.sm_count;
  if (grid <= 0) return ETHOS_OK;
  return launch_pdl(kern, dim3(grid), dim3(GemmCfg<Epi>::kThreads), GemmCfg<Epi>::kSmem, stream, ta, tb,
                    tc != nullptr ? *tc : ta, td != nullptr ? *td : ta, M, N, K, ksplit, epi, err, hold_unit);
}

template <class Epi, bool AMN = false, bool BMN = false>
int launch_gemm2sm(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const Epi& epi, int* err,
                   cudaStream_t stream, const DeviceInfo& dev, int ksplit = 1);

// D = A B^T.  N % 256 == 0 with an 8-warp epilogue runs on the 2-SM kernel
// (256 x 256 tiles per SM pair), everything else on k_gemm.
template <class Epi>
int gemm(const GemmOperand& a, const GemmOperand& b, int M, int N, int K, int ksplit, const Epi& epi, int* err,
         cudaStream_t stream, const DeviceInfo& dev) {
  if (M < 1 || N < 128 || N % 128 != 0 || K < 1) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (!a.mn_major && K % 8 != 0) return ETHOS_ERR_ALIGNMENT;
  if (!b.mn_major && K % 8 != 0) return ETHOS_ERR_ALIGNMENT;
  const bool wide = N % 256 == 0;
  constexpr bool kPairable = Epi::kEpiWarps == 8;
  const bool pair = wide && kPairable;
  CUtensorMap ta, tb;
  int st;
  if ((st = operand_tmap(&ta, a, M, K, 128)) != ETHOS_OK) return st;
  if ((st = operand_tmap(&tb, b, N, K, pair ? G2_BN / 2 : (wide ? 256 : 128))) != ETHOS_OK) return st;
  // never leave a K slice empty
  const int num_kb = (K + GEMM_BK - 1) / GEMM_BK;
  if (ksplit > num_kb) ksplit = num_kb;
  if (ksplit < 1) ksplit = 1;
  const int kpb = (num_kb + ksplit - 1) / ksplit;
  ksplit = (num_kb + kpb - 1) / kpb;
#define ETHOS_GEMM_CASE(AM, BM_)                                                                       \
  if (a.mn_major == AM && b.mn_major == BM_) {                                                        \
    if constexpr (kPairable) {                                                                        \
      if (pair) return launch_gemm2sm<Epi, AM, BM_>(ta, tb, M, N, K, epi, err, stream, dev, ksplit);  \
    }                                                                                                 \
    return wide ? launch_gemm_t<Epi, AM, BM_, 256>(ta, tb, M, N, K, ksplit, epi, err, stream, dev)     \
                : launch_gemm_t<Epi, AM, BM_, 128>(ta, tb, M, N, K, ksplit, epi, err, stream, dev);    \
  }
  ETHOS_GEMM_CASE(false, false)
  ETHOS_GEMM_CASE(true, false)
  ETHOS_GEMM_CASE(false, true)
  ETHOS_GEMM_CASE(true, true)
#undef ETHOS_GEMM_CASE
  return ETHOS_ERR_INVALID_ARG;
}

// Split count that fills the GPU for an accumulating GEMM with few tiles.
int auto_ksplit(int M, int N, int K, const DeviceInfo& dev) {
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * (N % 256 == 0 ? N / 256 : N / 128);
  const int num_kb = (K + GEMM_BK - 1) / GEMM_BK;
  int ks = dev.sm_count / (tiles > 0 ? tiles : 1);
  if (ks < 1) ks = 1;
  if (ks > num_kb) ks = num_kb;
  return ks;
}

// Clusters of two that can run at once for a 2-SM GEMM kernel (queried once
// per kernel and device: the SM-pair topology decides it, not the tile count).
int max_pair_clusters(const void* fn, int threads, int smem, const DeviceInfo& dev) {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return 0;
  static std::mutex mu;
  static const void* seen[64][8];
  static int val[64][8];
  static int nseen[64];
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < nseen[d]; ++i)
    if (seen[d][i] == fn) return val[d][i];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(dev.sm_count & ~1));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (nseen[d] < 8) {
    seen[d][nseen[d]] = fn;
    val[d][nseen[d]++] = n;
  }
  return n;
}

// 2-SM GEMM (k_gemm2sm).  A K-major `tb` has 128-row boxes (each CTA of a
// pair stages half of the 256-wide N tile), an MN-major one 64-column boxes.
// N % 256 == 0; ksplit > 1 requires an accumulating epilogue.
template <class Epi, bool AMN, bool BMN>
int launch_gemm2sm(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const Epi& epi, int* err,
                   cudaStream_t stream, const DeviceInfo& dev, int ksplit) {
  using Cfg = Gemm2Cfg<Epi>;
  auto kern = k_gemm2sm<Epi, AMN, BMN>;
  int st = smem_attr_once(reinterpret_cast<const void*>(kern), Cfg::kSmem);
  if (st != ETHOS_OK) return st;
  if (N % G2_BN != 0) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  const int units = ((M + 2 * G2_BM - 1) / (2 * G2_BM)) * (N / G2_BN) * ksplit;
  int pairs = max_pair_clusters(reinterpret_cast<const void*>(kern), Cfg::kThreads, Cfg::kSmem, dev);
  if (pairs <= 0) return ETHOS_ERR_CUDA;
  if (pairs > units) pairs = units;
  if (pairs <= 0) return ETHOS_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(static_cast<unsigned>(Cfg::kThreads));
  cfg.dynamicSmemBytes = static_cast<size_t>(Cfg::kSmem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel calls pdl_wait()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  count_launch();
  if (cudaLaunchKernelEx(&cfg, kern, ta, tb, M, N, K, ksplit, epi, err) != cudaSuccess) return ETHOS_ERR_CUDA;
  return launch_status();
}

// Forward-path GEMM: both operands K-major (tensor maps built by the caller).
template <class Epi>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const Epi& epi, int* err,
                cudaStream_t stream, const DeviceInfo& dev, const CUtensorMap* tc = nullptr,
                const CUtensorMap* td = nullptr) {
  return launch_gemm_t<Epi, false, false, 256>(ta, tb, M, N, K, 1, epi, err, stream, dev, -1, tc, td);
}

// ------------------------------------------------------- workspace layout --
struct Carve {
  char* base;
  size_t off = 0;
  size_t cap;
  template <class T>
  T* take(size_t count) {
    off = (off + 255) & ~static_cast<size_t>(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

struct FwdScratch {
  __half* table;
  __nv_bfloat16* qs;
  float2* colp;
  float* xp;
  __nv_bfloat16* hacc;
  float* qpre;
  float* save_bn;
  float* bn_part;
  int slabs;
};

void carve_forward(Carve& c, const ethos_dims& d, int bn_training, bool need_xp, bool need_hacc, bool need_qpre,
                   bool need_bn, bool need_table, FwdScratch* s) {
  const int64_t T = d.tokens, HQ = d.num_heads * d.d_query;
  s->table = need_table ? c.take<__half>(static_cast<size_t>(d.num_experts) * EX_DH) : nullptr;
  s->qs = c.take<__nv_bfloat16>(static_cast<size_t>(d.num_heads * 2 * T * d.d_query));
  s->colp = c.take<float2>(static_cast<size_t>(HQ));
  s->xp = need_xp ? c.take<float>(static_cast<size_t>(T * d.d_hidden)) : nullptr;
  s->hacc = need_hacc ? c.take<__nv_bfloat16>(static_cast<size_t>(T * d.d_hidden)) : nullptr;
  s->slabs = static_cast<int>((T + BN_ROWS_PER_SLAB - 1) / BN_ROWS_PER_SLAB);
  if (bn_training) {
    s->qpre = need_qpre ? c.take<float>(static_cast<size_t>(T * HQ)) : nullptr;
    s->save_bn = need_bn ? c.take<float>(static_cast<size_t>(2 * HQ)) : nullptr;
    s->bn_part = c.take<float>(static_cast<size_t>(s->slabs) * HQ * 2);
  } else {
    s->qpre = nullptr;
    s->save_bn = nullptr;
    s->bn_part = nullptr;
  }
}

int check_dims_impl(const ethos_dims* d) {
  if (d == nullptr) return ETHOS_ERR_INVALID_ARG;
  if (d->tokens < 1 || d->tokens > (int64_t(1) << 24)) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (d->d_latent != EX_DL || d->d_hidden != EX_DH) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  const int64_t R = d->num_heads * d->top_k;
  if (d->num_heads < 1 || R > EX_ROWS || R % 4 != 0) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (d->top_k != 4 && d->top_k != 8 && d->top_k != 16) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (d->num_sub_keys * d->num_sub_keys != d->num_experts) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (d->num_sub_keys % 32 != 0 || d->num_sub_keys > 512 || d->num_sub_keys < d->top_k)
    return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (d->d_query % 64 != 0 || d->d_query < 64) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (d->d_model % 256 != 0) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if ((d->num_heads * d->d_query + d->d_hidden) % 256 != 0) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if ((d->num_heads * d->d_query) % 256 != 0) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  return ETHOS_OK;
}

// Grid of the row-walking BatchNorm kernels: x covers the C / 8 column groups,
// y enough token rows to give every SM several blocks.
dim3 bn_rows_grid(int C, int T, int threads, const DeviceInfo& dev) {
  const int gx = (C / 8 + threads - 1) / threads;
  int gy = dev.sm_count * 8 / (gx > 0 ? gx : 1);
  if (gy < 1) gy = 1;
  if (gy > T) gy = T;
  if (gy > 65535) gy = 65535;
  return dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
}

// ------------------------------------------------------------ experts --
// Expert execution path: 1 = fused per-token (gather latents, expand on
// tcgen05, GELU in the epilogue), 2 = expert table (expand + GELU once per
// expert, then gather hidden rows per token), 3 = the table path on a table
// the caller built earlier (no expansion).  0 picks the table once the step
// makes at least one selection per expert on average.
int resolve_expert_path(const ethos_dims& d, int path) {
  if (path == 1) return 1;
  if (path == 3) return 3;
  if (path == 2) return d.num_heads * d.top_k >= 16 ? 2 : 1;
  const int64_t R = d.num_heads * d.top_k;
  const int64_t sel = d.tokens * R;
  return (sel >= d.num_experts && R >= 16) ? 2 : 1;
}

size_t expert_table_bytes(const ethos_dims& d) {
  return static_cast<size_t>(d.num_experts) * EX_DH * sizeof(__half);
}

// phase A: H = fp16(gelu(E @ W1^T)) [N, 512] (and, for training, G =
// fp16(gelu'(E @ W1^T)) alongside, for the backward)
int build_table(const ethos_dims& d, const void* latents, const void* w1, __half* table, __half* gtab, int* err,
                cudaStream_t stream, const DeviceInfo& dev) {
  const int N = static_cast<int>(d.num_experts);
  int st;
  CUtensorMap tm_e, tm_w1;
  if ((st = make_tmap_bf16(&tm_e, latents, N, EX_DL, 128)) != ETHOS_OK) return st;
  if ((st = make_tmap_bf16(&tm_w1, w1, EX_DH, EX_DL, 256)) != ETHOS_OK) return st;
  // the tables leave through TMA stores of 32-row x 64-column boxes (128-byte
  // swizzle), the layout the epilogue stages
  CUtensorMap tm_h;
  if ((st = make_tmap_bf16(&tm_h, table, N, EX_DH, 32, 0, 64, CU_TENSOR_MAP_DATA_TYPE_FLOAT16)) != ETHOS_OK) return st;
  if (gtab != nullptr) {  // training: G = gelu'(E W1^T) alongside, for the backward
    CUtensorMap tm_g;
    if ((st = make_tmap_bf16(&tm_g, gtab, N, EX_DH, 32, 0, 64, CU_TENSOR_MAP_DATA_TYPE_FLOAT16)) != ETHOS_OK)
      return st;
    return launch_gemm(tm_e, tm_w1, N, EX_DH, EX_DL, EpiGeluBwdF16{}, err, stream, dev, &tm_h, &tm_g);
  }
  return launch_gemm(tm_e, tm_w1, N, EX_DH, EX_DL, EpiGeluF16{}, err, stream, dev, &tm_h);
}

// phase B: per-token gather, dot, activation, weighted sum
int launch_gather(const __half* table, const int32_t* ids, const float* weights, const float* xp,
                  __nv_bfloat16* hacc, float* dot, int T, int R, int N, int* err, cudaStream_t stream,
                  const DeviceInfo& dev) {
  int blocks = (T + GATHER_WARPS - 1) / GATHER_WARPS;
  if (blocks > dev.sm_count) blocks = dev.sm_count;
  return launch_pdl(k_expert_gather, dim3(blocks), dim3(GATHER_THREADS), GATHER_SMEM_BYTES, stream, table, ids,
                    weights, xp, hacc, dot, T, R, N, err);
}

int run_experts(const ethos_dims& d, int path, const void* latents, const void* w1, const int32_t* ids,
                const float* weights, const float* xp, __nv_bfloat16* hacc, float* dot, __half* table, int* err,
                cudaStream_t stream, const DeviceInfo& dev, void* const* ev = nullptr, __half* gtab = nullptr) {
  const int T = static_cast<int>(d.tokens);
  const int R = static_cast<int>(d.num_heads * d.top_k);
  const int N = static_cast<int>(d.num_experts);
  int st;
  if (path == 1) {
    CUtensorMap tm_w1;
    if ((st = make_tmap_bf16(&tm_w1, w1, EX_DH, EX_DL, 256)) != ETHOS_OK) return st;
    ExpertFwdArgs ea;
    ea.latents = static_cast<const __nv_bfloat16*>(latents);
    ea.ids = ids;
    ea.w = weights;
    ea.xp = xp;
    ea.hacc = hacc;
    ea.save_dot = dot;
    ea.T = T;
    ea.R = R;
    ea.N = N;
    const int grid = T < dev.sm_count ? T : dev.sm_count;
    mark(ev, ETHOS_STAGE_EXPERT_TABLE, stream);
    count_launch();
    k_expert_fwd<<<grid, EX_THREADS, EX_SMEM_BYTES, stream>>>(tm_w1, ea, err);
    return launch_status();
  }
  if (path == 3) {  // the caller's table: phase A is skipped
    mark(ev, ETHOS_STAGE_EXPERT_TABLE, stream);
    return launch_gather(table, ids, weights, xp, hacc, dot, T, R, N, err, stream, dev);
  }
  if ((st = build_table(d, latents, w1, table, gtab, err, stream, dev)) != ETHOS_OK) return st;
  mark(ev, ETHOS_STAGE_EXPERT_TABLE, stream);
  return launch_gather(table, ids, weights, xp, hacc, dot, T, R, N, err, stream, dev);
}

template <int TOPK>
int launch_score(const CUtensorMap& ta, const CUtensorMap& tb, const RouterGeom& g, int32_t* ids, float* w,
                 int* err, cudaStream_t stream, const DeviceInfo& dev) {
  const int items = g.H * ((g.T + 127) / 128);
  const int grid = items < dev.sm_count ? items : dev.sm_count;
  return launch_pdl(k_score_topk<TOPK>, dim3(grid), dim3(ROUTER_THREADS), ROUTER_SMEM_BYTES, stream, ta, tb, g, ids,
                    w, err);
}

int run_score(const CUtensorMap& ta, const CUtensorMap& tb, const RouterGeom& g, int top_k, int32_t* ids,
              float* w, int* err, cudaStream_t stream, const DeviceInfo& dev) {
  switch (top_k) {
    case 4: return launch_score<4>(ta, tb, g, ids, w, err, stream, dev);
    case 8: return launch_score<8>(ta, tb, g, ids, w, err, stream, dev);
    case 16: return launch_score<16>(ta, tb, g, ids, w, err, stream, dev);
    default: return ETHOS_ERR_UNSUPPORTED_SHAPE;
  }
}

// Router part shared by ethos_layer_forward and ethos_router_forward:
// projection GEMM (queries, plus x_proj when with_xp), BatchNorm, scoring and
// top-k.
// `qs` is the split-bf16 scoring operand [2][H][T][dq] (scratch, or the
// caller's save buffer).  With keep_qpre the projection always writes the
// pre-BatchNorm queries (fp32) and normalises them in a second pass, so the
// backward pass has them in both BatchNorm modes.
int router_core(const ethos_dims& d, const void* x, const void* w_cat, float* bn, float bn_eps, float bn_momentum,
                int bn_training, const void* key_cat, int32_t* ids, float* weights, bool with_xp, float* xp_out,
                const FwdScratch& s, __nv_bfloat16* qs, float* qpre, bool keep_qpre, float* save_bn, int* err,
                cudaStream_t stream, const DeviceInfo& dev, void* const* ev = nullptr) {
  const int T = static_cast<int>(d.tokens);
  const int HQ = static_cast<int>(d.num_heads * d.d_query);
  const int dq = static_cast<int>(d.d_query);
  const int dh = static_cast<int>(d.d_hidden);
  const int ncat = with_xp ? HQ + dh : HQ;
  const bool two_pass = bn_training || keep_qpre;
  CUtensorMap tm_x, tm_w, tm_q, tm_k;
  int st;
  if ((st = make_tmap_bf16(&tm_x, x, T, d.d_model, 128)) != ETHOS_OK) return st;
  if ((st = make_tmap_bf16(&tm_w, w_cat, ncat, d.d_model, G2_BN / 2)) != ETHOS_OK) return st;
  if ((st = make_tmap_bf16(&tm_q, qs, static_cast<int64_t>(d.num_heads) * 2 * T, dq, 128, 0, ROUTER_KB)) != ETHOS_OK)
    return st;
  const int box_keys = d.num_sub_keys < 256 ? static_cast<int>(d.num_sub_keys) : 256;
  if ((st = make_tmap_bf16(&tm_k, key_cat, 2 * d.num_sub_keys, dq, box_keys, 0, ROUTER_KB)) != ETHOS_OK) return st;

  const int cb = 256;
  if (!bn_training) {
    if ((st = launch_pdl(k_bn_eval_colp, dim3((HQ + cb - 1) / cb), dim3(cb), 0, stream, bn, HQ, bn_eps,
                         two_pass ? 1 : 0, s.colp)) != ETHOS_OK)
      return st;
  }
  EpiProj epi;
  epi.M = T;
  epi.HQ = HQ;
  epi.dq = dq;
  epi.dh = dh;
  epi.mode = two_pass ? 1 : 0;
  epi.bias = bn;
  epi.colp = s.colp;
  epi.qs = qs;
  epi.qpre = qpre;
  epi.xp = xp_out;
  epi.part = nullptr;
  epi.ldp = 0;
  if ((st = launch_gemm2sm(tm_x, tm_w, T, ncat, static_cast<int>(d.d_model), epi, err, stream, dev)) != ETHOS_OK)
    return st;
  mark(ev, ETHOS_STAGE_PROJECTION, stream);
  if (two_pass) {
    if (bn_training) {
      dim3 grid_p((HQ + cb - 1) / cb, s.slabs);
      count_launch();
      k_bn_partial<<<grid_p, cb, 0, stream>>>(qpre, T, HQ, s.bn_part);
      count_launch();
      k_bn_finalize<<<(HQ + cb - 1) / cb, cb, 0, stream>>>(qpre, s.bn_part, T, HQ, s.slabs, bn + HQ, bn + 2 * HQ,
                                                           bn + 3 * HQ, bn + 4 * HQ, bn_eps, bn_momentum, save_bn,
                                                           s.colp);
    }
    count_launch();
    k_bn_apply<<<bn_rows_grid(HQ, T, cb, dev), cb, 0, stream>>>(qpre, s.colp, T, static_cast<int>(d.num_heads),
                                                                 dq, qs);
    if ((st = launch_status()) != ETHOS_OK) return st;
  }
  mark(ev, ETHOS_STAGE_BATCHNORM, stream);
  RouterGeom g;
  g.T = T;
  g.H = static_cast<int>(d.num_heads);
  g.K = static_cast<int>(d.num_sub_keys);
  g.KA = dq;
  g.a_stride_h = T;
  g.a_stride_p = static_cast<int>(d.num_heads) * T;
  g.a_col_p = 0;
  g.split = 1;
  st = run_score(tm_q, tm_k, g, static_cast<int>(d.top_k), ids, weights, err, stream, dev);
  mark(ev, ETHOS_STAGE_TOPK, stream);
  return st;
}

// ------------------------------------------------------- backward scratch --
struct BwdScratch {
  __half* htab;
  __half* gtab;
  float* dhacc;
  float* dw;
  float* ca;
  float* cd;
  float* dxp;
  __nv_bfloat16* du;
  int* cnt;
  int* offs;
  int* cursor;
  int* bsums;
  int* total;
  int* perm;
  __nv_bfloat16* dP;
  __nv_bfloat16* dqhat;  // [T][HQ] dq^ (bf16: feeds BatchNorm's backward only)
  __nv_bfloat16* dS;
  __nv_bfloat16* gx;
  float* part;
  float* coef;
  float* stats;
  __nv_bfloat16* dy16;
  int slabs;
};

void carve_backward(Carve& c, const ethos_dims& d, BwdScratch* s) {
  const int64_t T = d.tokens, N = d.num_experts, R = d.num_heads * d.top_k, HQ = d.num_heads * d.d_query;
  s->htab = c.take<__half>(static_cast<size_t>(N * EX_DH));
  s->gtab = c.take<__half>(static_cast<size_t>(N * EX_DH));
  s->dhacc = c.take<float>(static_cast<size_t>(T * EX_DH));
  s->dw = c.take<float>(static_cast<size_t>(T * R));
  s->ca = c.take<float>(static_cast<size_t>(T * R));
  s->cd = c.take<float>(static_cast<size_t>(T * R));
  s->dxp = c.take<float>(static_cast<size_t>(T * EX_DH));
  s->du = c.take<__nv_bfloat16>(static_cast<size_t>(T * (HQ + EX_DH)));
  s->cnt = c.take<int>(static_cast<size_t>(N));
  s->offs = c.take<int>(static_cast<size_t>(N));
  s->cursor = c.take<int>(static_cast<size_t>(N));
  s->bsums = c.take<int>(1024);
  s->total = c.take<int>(4);
  s->perm = c.take<int>(static_cast<size_t>(T * R));
  s->dP = c.take<__nv_bfloat16>(static_cast<size_t>(N * EX_DH));
  s->dqhat = c.take<__nv_bfloat16>(static_cast<size_t>(T * HQ));
  s->dS = c.take<__nv_bfloat16>(static_cast<size_t>(d.num_heads * 2 * T * d.num_sub_keys));
  s->gx = c.take<__nv_bfloat16>(static_cast<size_t>(T * 2 * EX_DH));
  s->slabs = static_cast<int>((T + BN_ROWS_PER_SLAB - 1) / BN_ROWS_PER_SLAB);
  s->part = c.take<float>(static_cast<size_t>(s->slabs) * HQ * 2);
  s->coef = c.take<float>(static_cast<size_t>(4 * HQ));
  s->stats = c.take<float>(static_cast<size_t>(2 * HQ));
  s->dy16 = c.take<__nv_bfloat16>(static_cast<size_t>(T * d.d_model));
}

__global__ void k_f32_to_bf16(const float* __restrict__ in, int64_t n, __nv_bfloat16* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(in[i]);
}

template <int TOPK>
int launch_router_bwd(const ethos_dims& d, const int32_t* ids, const float* w, const float* dw,
                      const __nv_bfloat16* keys, int64_t key_ld, __nv_bfloat16* dqhat, __nv_bfloat16* dS,
                      cudaStream_t stream,
                      const DeviceInfo& dev) {
  const int TH = static_cast<int>(d.tokens * d.num_heads);
  int blocks = (TH + 7) / 8;
  if (blocks > dev.sm_count * 8) blocks = dev.sm_count * 8;
  count_launch();
  k_router_bwd<TOPK><<<blocks, 256, 0, stream>>>(ids, w, dw, keys, key_ld, dqhat, dS, static_cast<int>(d.tokens),
                                                  static_cast<int>(d.num_heads), static_cast<int>(d.num_sub_keys),
                                                  static_cast<int>(d.d_query / 2));
  return launch_status();
}

// Scratch of ethos_expert_backward: the expert half of BwdScratch plus a
// [T, dh] bf16 operand row block for dxp (the kernel writes it as a GEMM
// operand; only the fp32 dxp is returned).
void carve_expert_backward(Carve& c, const ethos_dims& d, BwdScratch* s) {
  const int64_t T = d.tokens, N = d.num_experts, R = d.num_heads * d.top_k;
  *s = BwdScratch{};
  s->htab = c.take<__half>(static_cast<size_t>(N * EX_DH));
  s->gtab = c.take<__half>(static_cast<size_t>(N * EX_DH));
  s->ca = c.take<float>(static_cast<size_t>(T * R));
  s->cd = c.take<float>(static_cast<size_t>(T * R));
  s->du = c.take<__nv_bfloat16>(static_cast<size_t>(T * EX_DH));
  s->cnt = c.take<int>(static_cast<size_t>(N));
  s->offs = c.take<int>(static_cast<size_t>(N));
  s->cursor = c.take<int>(static_cast<size_t>(N));
  s->bsums = c.take<int>(1024);
  s->total = c.take<int>(4);
  s->perm = c.take<int>(static_cast<size_t>(T * R));
  s->dP = c.take<__nv_bfloat16>(static_cast<size_t>(N * EX_DH));
  s->gx = c.take<__nv_bfloat16>(static_cast<size_t>(T * 2 * EX_DH));
}

// Scratch of ethos_router_backward: the router half of BwdScratch, the dq
// operand [T, H*dq] bf16, and the recomputed normalised queries qs with
// their per-column affine.
struct RouterBwdExtra {
  __nv_bfloat16* qs;  // [2][H][T][dq]
  float2* colp;       // [H*dq]
};

void carve_router_backward(Carve& c, const ethos_dims& d, BwdScratch* s, RouterBwdExtra* x) {
  const int64_t T = d.tokens, HQ = d.num_heads * d.d_query;
  *s = BwdScratch{};
  s->du = c.take<__nv_bfloat16>(static_cast<size_t>(T * HQ));
  s->dqhat = c.take<__nv_bfloat16>(static_cast<size_t>(T * HQ));
  s->dS = c.take<__nv_bfloat16>(static_cast<size_t>(d.num_heads * 2 * T * d.num_sub_keys));
  s->slabs = static_cast<int>((T + BN_ROWS_PER_SLAB - 1) / BN_ROWS_PER_SLAB);
  s->part = c.take<float>(static_cast<size_t>(s->slabs) * HQ * 2);
  s->coef = c.take<float>(static_cast<size_t>(4 * HQ));
  s->stats = c.take<float>(static_cast<size_t>(2 * HQ));
  x->qs = c.take<__nv_bfloat16>(static_cast<size_t>(2 * T * HQ));
  x->colp = c.take<float2>(static_cast<size_t>(HQ));
}

// Inputs and outputs of the expert half of the backward.
struct ExpertBwdIO {
  const void* latents;
  const void* w1;
  const int32_t* ids;
  const float* weights;
  const float* xp;     // fp32 [T, dh]
  const float* dot;    // fp32 [T, R]
  const float* dhacc;  // fp32 [T, dh]
  const void* htab;    // fp16 [N, dh] or NULL (then built here with gtab)
  const void* gtab;
  float* dxp;          // fp32 [T, dh] out
  __nv_bfloat16* du;   // bf16 copy of dxp at du[t * ldu + du_off + j]
  int64_t ldu;
  int du_off;
  float* dw;           // fp32 [T, R] out: dL/d(routing weight)
  float* d_latents;
  float* d_w1;
};

// Expert half of the backward (the gradients autograd takes through the
// expert loop of model.py:306-336 given hacc's gradient): per-selection
// weight gradients and dxp, then per-expert dP by a counting sort of the
// selections, dE = dP W1 and dW1 = dP^T E.  Scratch from s: htab / gtab
// (when io.htab is NULL), ca, cd, gx, the sort arrays and dP.
int expert_bwd_core(const ethos_dims& d, const ExpertBwdIO& io, const BwdScratch& s, int* dev_err,
                    cudaStream_t sm, const DeviceInfo& dev) {
  const int T = static_cast<int>(d.tokens), N = static_cast<int>(d.num_experts);
  const int R = static_cast<int>(d.num_heads * d.top_k);
  const int cb = 256;
  const int eblocks = dev.sm_count * 8;
  int st;
  if (cudaMemsetAsync(io.d_w1, 0, sizeof(float) * EX_DH * EX_DL, sm) != cudaSuccess) return ETHOS_ERR_CUDA;
  if (cudaMemsetAsync(s.cnt, 0, sizeof(int) * N, sm) != cudaSuccess) return ETHOS_ERR_CUDA;
  // per-expert tables H = gelu(E W1^T), G = gelu'(E W1^T) (fp16), unless the
  // forward kept them
  const __half* htab_ = io.htab ? static_cast<const __half*>(io.htab) : s.htab;
  const __half* gtab_ = io.gtab ? static_cast<const __half*>(io.gtab) : s.gtab;
  if (io.htab == nullptr) {
    if ((st = build_table(d, io.latents, io.w1, s.htab, s.gtab, dev_err, sm, dev)) != ETHOS_OK) return st;
  }
  // per token: dw, a, ddot per selection; dxp (fp32 + bf16 operand)
  {
    if (BGATHER_STAGES - 1 < R / GATHER_ROWS) {  // one dhacc / xp buffer per warp
      constexpr int bytes = bgather_smem_bytes(BGATHER_WARPS, BGATHER_STAGES, 1);
      auto kern = k_expert_bwd_gather<BGATHER_WARPS, BGATHER_STAGES, 1>;
      if ((st = smem_attr_once(reinterpret_cast<const void*>(kern), bytes)) != ETHOS_OK) return st;
      int blocks = (T + BGATHER_WARPS - 1) / BGATHER_WARPS;
      if (blocks > dev.sm_count) blocks = dev.sm_count;
      count_launch();
      kern<<<blocks, BGATHER_WARPS * 32, bytes, sm>>>(htab_, io.ids, io.weights, io.dot, io.dhacc, io.dw, s.ca, s.cd,
                                                      io.dxp, io.du, io.ldu, io.du_off, io.xp, s.gx, T, R, N,
                                                      dev_err);
    } else {  // R = 4: double buffers, 2 stages
      constexpr int W = BGATHER_SMALL_R_WARPS;
      constexpr int bytes = bgather_smem_bytes(W, 2, 2);
      auto kern = k_expert_bwd_gather<W, 2, 2>;
      if ((st = smem_attr_once(reinterpret_cast<const void*>(kern), bytes)) != ETHOS_OK) return st;
      int blocks = (T + W - 1) / W;
      if (blocks > dev.sm_count) blocks = dev.sm_count;
      count_launch();
      kern<<<blocks, W * 32, bytes, sm>>>(htab_, io.ids, io.weights, io.dot, io.dhacc, io.dw, s.ca, s.cd, io.dxp,
                                          io.du, io.ldu, io.du_off, io.xp, s.gx, T, R, N, dev_err);
    }
    if ((st = launch_status()) != ETHOS_OK) return st;
  }
  // selections grouped by expert (counting sort)
  {
    const int64_t nsel = static_cast<int64_t>(T) * R;
    count_launch();
    k_count_experts<<<eblocks, cb, 0, sm>>>(io.ids, nsel, N, s.cnt, dev_err);
    const int nblk = (N + 1023) / 1024;
    if (nblk > 1024) return ETHOS_ERR_UNSUPPORTED_SHAPE;
    count_launch();
    k_scan_blocks<<<nblk, 1024, 0, sm>>>(s.cnt, N, s.offs, s.bsums);
    count_launch();
    k_scan_sums<<<1, 1024, 0, sm>>>(s.bsums, nblk, s.total);
    count_launch();
    k_scan_add<<<nblk, 1024, 0, sm>>>(s.offs, N, s.bsums, s.cursor);
    count_launch();
    k_scatter_experts<<<eblocks, cb, 0, sm>>>(io.ids, nsel, N, s.cursor, s.perm);
    if ((st = launch_status()) != ETHOS_OK) return st;
  }
  // dP[e] = G[e] * sum over e's selections of (a dhacc_t + ddot xp_t)
  count_launch();
  k_expert_dP<<<eblocks, 256, 0, sm>>>(s.offs, s.perm, s.total, s.ca, s.cd, s.gx, gtab_, s.dP, N, R);
  if ((st = launch_status()) != ETHOS_OK) return st;
  // dE = dP W1       (W1 read in place, MN-major)
  {
    EpiStoreF32 e;
    e.out = io.d_latents;
    e.ldo = EX_DL;
    e.M = N;
    e.scale = 1.0f;
    e.accumulate = 0;
    if ((st = gemm(GemmOperand{s.dP, EX_DH, false}, GemmOperand{io.w1, EX_DL, true}, N, EX_DL, EX_DH, 1, e, dev_err,
                   sm, dev)) != ETHOS_OK)
      return st;
  }
  // dW1 = dP^T E     (both read in place, MN-major; split-K over experts)
  {
    EpiAtomicF32 e;
    e.out = io.d_w1;
    e.ldo = EX_DL;
    e.M = EX_DH;
    e.scale = 1.0f;
    if ((st = gemm(GemmOperand{s.dP, EX_DH, true}, GemmOperand{io.latents, EX_DL, true}, EX_DH, EX_DL, N,
                   auto_ksplit(EX_DH, EX_DL, N, dev), e, dev_err, sm, dev)) != ETHOS_OK)
      return st;
  }
  return ETHOS_OK;
}

// Inputs and outputs of the router half of the backward.
struct RouterBwdIO {
  int bn_training;
  float bn_eps;
  const float* bn;
  const void* key_cat;
  const int32_t* ids;
  const float* weights;
  const float* dw;        // fp32 [T, R]: dL/d(routing weight)
  const float* qpre;      // fp32 [T, H*dq]
  const float* save_bn;   // fp32 [2, H*dq] (training) or NULL
  const void* qs;         // bf16 [2][H][T][dq] normalised queries (hi | lo)
  __nv_bfloat16* du;      // dq (bf16) out at du[t * ldu + c], c < H*dq
  int64_t ldu;
  float* d_bn;
  float* d_keys;
};

// Router half of the backward (model.py:208-254 under autograd): softmax
// backward into the selected grid scores, the dense sub-key score gradient
// dS and dq^, dK = dS^T q^, then BatchNorm's backward into dq and the
// bias / gamma / beta gradients.  Scratch from s: dqhat, dS, part, coef,
// stats.
int router_bwd_core(const ethos_dims& d, const RouterBwdIO& io, const BwdScratch& s, int* dev_err,
                    cudaStream_t sm, const DeviceInfo& dev) {
  const int T = static_cast<int>(d.tokens), H = static_cast<int>(d.num_heads);
  const int dq = static_cast<int>(d.d_query), HQ = H * dq, K = static_cast<int>(d.num_sub_keys), half = dq / 2;
  const int cb = 256;
  int st;
  if (cudaMemsetAsync(io.d_keys, 0, sizeof(float) * 2 * K * half, sm) != cudaSuccess) return ETHOS_ERR_CUDA;
  // softmax backward, dq^ and the dense sub-key score gradient dS (k_router_bwd
  // writes every row of dS, zeros included)
  const __nv_bfloat16* keys = static_cast<const __nv_bfloat16*>(io.key_cat);
  switch (d.top_k) {
    case 4: st = launch_router_bwd<4>(d, io.ids, io.weights, io.dw, keys, dq, s.dqhat, s.dS, sm, dev); break;
    case 8: st = launch_router_bwd<8>(d, io.ids, io.weights, io.dw, keys, dq, s.dqhat, s.dS, sm, dev); break;
    default: st = launch_router_bwd<16>(d, io.ids, io.weights, io.dw, keys, dq, s.dqhat, s.dS, sm, dev); break;
  }
  if (st != ETHOS_OK) return st;
  // dK_p = dS_p^T q^_p over all heads and tokens (q^ = hi part of qs; both
  // [2][H][T][.] so the (h, t) rows of a half are contiguous)
  for (int p = 0; p < 2; ++p) {
    EpiAtomicF32 e;
    e.out = io.d_keys + static_cast<int64_t>(p) * K * half;
    e.ldo = half;
    e.M = K;
    e.scale = 1.0f;
    const __nv_bfloat16* dSp = s.dS + static_cast<int64_t>(p) * H * T * K;
    const __nv_bfloat16* qh = static_cast<const __nv_bfloat16*>(io.qs) + static_cast<int64_t>(p) * H * T * dq;
    const int KK = H * T;
    if ((st = gemm(GemmOperand{dSp, K, true}, GemmOperand{qh, dq, true}, K, half, KK, auto_ksplit(K, half, KK, dev),
                   e, dev_err, sm, dev)) != ETHOS_OK)
      return st;
  }
  // BatchNorm backward -> dq (bf16 into du[:, :HQ]), dbias, dgamma, dbeta
  const float* mean = io.save_bn;
  const float* invstd = io.save_bn ? io.save_bn + HQ : nullptr;
  if (!io.bn_training) {
    count_launch();
    k_bn_eval_stats<<<(HQ + cb - 1) / cb, cb, 0, sm>>>(io.bn, HQ, io.bn_eps, s.stats, s.stats + HQ);
    mean = s.stats;
    invstd = s.stats + HQ;
  }
  dim3 grid_p((HQ / 2 + cb - 1) / cb, s.slabs);
  count_launch();
  k_bn_bwd_partial_bf16<<<grid_p, cb, 0, sm>>>(s.dqhat, io.qpre, mean, invstd, T, HQ, s.part);
  count_launch();
  k_bn_bwd_finalize<<<(HQ + cb - 1) / cb, cb, 0, sm>>>(s.part, s.slabs, HQ, T, io.bn_training, io.bn + HQ, mean,
                                                      invstd, io.d_bn + HQ, io.d_bn + 2 * HQ, io.d_bn, s.coef);
  count_launch();
  k_bn_bwd_apply<<<bn_rows_grid(HQ, T, cb, dev), cb, 0, sm>>>(s.dqhat, io.qpre, reinterpret_cast<const float4*>(s.coef),
                                                              T, HQ, io.du, io.ldu);
  return launch_status();
}

}  // namespace

// =================================================================== ABI ==
extern "C" {

int ethos_abi_version(void) { return kAbiVersion; }

uint64_t ethos_launch_count(void) { return g_launch_count.load(std::memory_order_relaxed); }

const char* ethos_status_string(int status) {
  switch (status) {
    case ETHOS_OK: return "ok";
    case ETHOS_ERR_INVALID_ARG: return "invalid argument";
    case ETHOS_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case ETHOS_ERR_ALIGNMENT: return "pointer or row pitch not 16-byte aligned";
    case ETHOS_ERR_WORKSPACE: return "workspace too small";
    case ETHOS_ERR_CUDA: return "CUDA runtime error";
    case ETHOS_ERR_TENSOR_MAP: return "tensor map encoding failed";
    case ETHOS_ERR_NO_DEVICE: return "no sm_100 device is current";
    case ETHOS_ERR_SCRATCH_LIMIT: return "request exceeds the static scratch of the no-allocation entry point";
    case ETHOS_ERR_ID_OUT_OF_RANGE: return "expert id out of range (device)";
    default:
      if (status >= ETHOS_ERR_TIMEOUT_BASE) return "bounded device wait timed out";
      return "unknown status";
  }
}

int ethos_read_device_error(int* dev_err, int* host_code, int reset, void* stream) {
  if (dev_err == nullptr || host_code == nullptr) return ETHOS_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  if (cudaMemcpyAsync(&v, dev_err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return ETHOS_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return ETHOS_ERR_CUDA;
  *host_code = v;
  if (reset && v != 0) {
    if (cudaMemsetAsync(dev_err, 0, sizeof(int), s) != cudaSuccess) return ETHOS_ERR_CUDA;
  }
  return ETHOS_OK;
}

int ethos_check_dims(const ethos_dims* dims) { return check_dims_impl(dims); }

size_t ethos_forward_workspace_size(const ethos_dims* dims, int bn_training, int expert_path) {
  if (check_dims_impl(dims) != ETHOS_OK) return 0;
  Carve c{nullptr, 0, 0};
  FwdScratch s;
  carve_forward(c, *dims, bn_training, true, true, true, true, resolve_expert_path(*dims, expert_path) == 2, &s);
  return c.off + 256;
}

size_t ethos_expert_workspace_size(const ethos_dims* dims, int expert_path) {
  if (check_dims_impl(dims) != ETHOS_OK) return 0;
  return resolve_expert_path(*dims, expert_path) >= 2 ? expert_table_bytes(*dims) + 256 : 256;
}

int ethos_expert_table_build(const ethos_dims* dims, const void* latents, const void* w1, void* htab, void* gtab,
                             int* dev_err, void* stream) {
  int st = check_dims_impl(dims);
  if (st != ETHOS_OK) return st;
  if (!latents || !w1 || !htab || !dev_err) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(latents) || !aligned16(w1) || !aligned16(htab) || (gtab && !aligned16(gtab)))
    return ETHOS_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  return build_table(*dims, latents, w1, static_cast<__half*>(htab), static_cast<__half*>(gtab), dev_err,
                     static_cast<cudaStream_t>(stream), *dev);
}

int ethos_layer_forward(const ethos_dims* dims, const void* x, const void* w_cat, float* bn, float bn_eps,
                        float bn_momentum, int bn_training, const void* key_cat, const void* latents,
                        const void* w1, const void* wv, int expert_path, void* y, int32_t* ids, float* weights,
                        float* save_xp, void* save_hacc, float* save_dot, float* save_qpre, float* save_bn,
                        void* save_qs, void* save_htab, void* save_gtab, void* workspace, size_t workspace_bytes,
                        int* dev_err, void* const* stage_events, void* stream) {
  int st = check_dims_impl(dims);
  if (st != ETHOS_OK) return st;
  if (!x || !w_cat || !bn || !key_cat || !latents || !w1 || !wv || !y || !ids || !weights || !workspace || !dev_err)
    return ETHOS_ERR_INVALID_ARG;
  if (expert_path < 0 || expert_path > 3) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_cat) || !aligned16(bn) || !aligned16(key_cat) || !aligned16(latents) ||
      !aligned16(w1) || !aligned16(wv) || !aligned16(y) || !aligned16(ids) || !aligned16(weights) ||
      !aligned16(workspace) || (save_xp && !aligned16(save_xp)) || (save_hacc && !aligned16(save_hacc)) ||
      (save_qpre && !aligned16(save_qpre)) || (save_qs && !aligned16(save_qs)) ||
      (save_htab && !aligned16(save_htab)) || (save_gtab && !aligned16(save_gtab)))
    return ETHOS_ERR_ALIGNMENT;
  if (expert_path == 3) {  // save_htab is the caller's table, read only
    if (save_htab == nullptr || save_gtab != nullptr) return ETHOS_ERR_INVALID_ARG;
    if (dims->num_heads * dims->top_k < 16) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  } else if ((save_htab == nullptr) != (save_gtab == nullptr)) {
    return ETHOS_ERR_INVALID_ARG;
  }
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  const ethos_dims& d = *dims;
  const int path = resolve_expert_path(d, expert_path);
  const bool keep_tables = save_htab != nullptr && path >= 2;
  if (workspace_bytes < ethos_forward_workspace_size(dims, bn_training, path)) return ETHOS_ERR_WORKSPACE;
  cudaStream_t stream_ = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<char*>(workspace), 0, workspace_bytes};
  FwdScratch s;
  carve_forward(c, d, bn_training, save_xp == nullptr, save_hacc == nullptr, save_qpre == nullptr,
                save_bn == nullptr, path == 2, &s);
  float* xp = save_xp ? save_xp : s.xp;
  __nv_bfloat16* hacc = save_hacc ? static_cast<__nv_bfloat16*>(save_hacc) : s.hacc;
  float* qpre = save_qpre ? save_qpre : s.qpre;
  float* sbn = save_bn ? save_bn : s.save_bn;
  const int T = static_cast<int>(d.tokens);
  void* const* ev = stage_events;
  mark(ev, ETHOS_STAGE_START, stream_);
  __nv_bfloat16* qs = save_qs ? static_cast<__nv_bfloat16*>(save_qs) : s.qs;
  if ((st = router_core(d, x, w_cat, bn, bn_eps, bn_momentum, bn_training, key_cat, ids, weights, true, xp, s, qs,
                        qpre, save_qpre != nullptr, sbn, dev_err, stream_, *dev, ev)) != ETHOS_OK)
    return st;
  if ((st = run_experts(d, path, latents, w1, ids, weights, xp, hacc, save_dot,
                        keep_tables ? static_cast<__half*>(save_htab) : s.table, dev_err, stream_, *dev, ev,
                        keep_tables ? static_cast<__half*>(save_gtab) : nullptr)) != ETHOS_OK)
    return st;
  mark(ev, ETHOS_STAGE_EXPERTS, stream_);

  // y = hacc @ W_v / H   (model.py:332-341)
  CUtensorMap tm_h, tm_v;
  if ((st = make_tmap_bf16(&tm_h, hacc, T, EX_DH, 128)) != ETHOS_OK) return st;
  if ((st = make_tmap_bf16(&tm_v, wv, d.d_model, EX_DH, 256)) != ETHOS_OK) return st;
  EpiStoreBF16 ey;
  ey.out = static_cast<__nv_bfloat16*>(y);
  ey.ldo = d.d_model;
  ey.M = T;
  ey.scale = 1.0f / static_cast<float>(d.num_heads);
  st = launch_gemm(tm_h, tm_v, T, static_cast<int>(d.d_model), EX_DH, ey, dev_err, stream_, *dev);
  mark(ev, ETHOS_STAGE_END, stream_);
  return st;
}

int ethos_router_forward(const ethos_dims* dims, const void* x, const void* w_cat, float* bn, float bn_eps,
                         float bn_momentum, int bn_training, const void* key_cat, int32_t* ids, float* weights,
                         float* save_qpre, float* save_bn, void* workspace, size_t workspace_bytes, int* dev_err,
                         void* stream) {
  int st = check_dims_impl(dims);
  if (st != ETHOS_OK) return st;
  if (!x || !w_cat || !bn || !key_cat || !ids || !weights || !workspace || !dev_err) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_cat) || !aligned16(bn) || !aligned16(key_cat) || !aligned16(ids) ||
      !aligned16(weights) || !aligned16(workspace) || (save_qpre && !aligned16(save_qpre)))
    return ETHOS_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  if (workspace_bytes < ethos_forward_workspace_size(dims, bn_training, 1)) return ETHOS_ERR_WORKSPACE;
  Carve c{static_cast<char*>(workspace), 0, workspace_bytes};
  FwdScratch s;
  carve_forward(c, *dims, bn_training, false, false, save_qpre == nullptr, save_bn == nullptr, false, &s);
  float* qpre = save_qpre ? save_qpre : s.qpre;
  float* sbn = save_bn ? save_bn : s.save_bn;
  // with save_qpre the pre-BatchNorm queries are kept in eval mode too (the
  // two-pass form), as ethos_router_backward needs them
  return router_core(*dims, x, w_cat, bn, bn_eps, bn_momentum, bn_training, key_cat, ids, weights, false, nullptr,
                     s, s.qs, qpre, save_qpre != nullptr, sbn, dev_err, static_cast<cudaStream_t>(stream), *dev);
}

int ethos_expert_forward(const ethos_dims* dims, int expert_path, const void* latents, const void* w1,
                         const int32_t* ids, const float* weights, const float* xp, void* hacc, float* dot,
                         void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
  int st = check_dims_impl(dims);
  if (st != ETHOS_OK) return st;
  if (!latents || !w1 || !ids || !weights || !xp || !hacc || !dev_err) return ETHOS_ERR_INVALID_ARG;
  if (expert_path < 0 || expert_path > 3) return ETHOS_ERR_INVALID_ARG;
  if (expert_path == 3 && dims->num_heads * dims->top_k < 16) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (!aligned16(latents) || !aligned16(w1) || !aligned16(ids) || !aligned16(weights) || !aligned16(xp) ||
      !aligned16(hacc) || (workspace && !aligned16(workspace)))
    return ETHOS_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  const int path = resolve_expert_path(*dims, expert_path);
  if (path >= 2 && (workspace == nullptr || workspace_bytes < expert_table_bytes(*dims)))
    return ETHOS_ERR_WORKSPACE;
  return run_experts(*dims, path, latents, w1, ids, weights, xp, static_cast<__nv_bfloat16*>(hacc), dot,
                     static_cast<__half*>(workspace), dev_err, static_cast<cudaStream_t>(stream), *dev);
}

int ethos_product_key_topk(const ethos_dims* dims, const void* q, const void* keys, int32_t* ids, float* weights,
                           int* dev_err, void* stream) {
  if (dims == nullptr || !q || !keys || !ids || !weights || !dev_err) return ETHOS_ERR_INVALID_ARG;
  const ethos_dims& d = *dims;
  if (d.tokens < 1 || d.num_heads < 1) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (d.top_k != 4 && d.top_k != 8 && d.top_k != 16) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (d.num_sub_keys % 32 != 0 || d.num_sub_keys > 512 || d.num_sub_keys < d.top_k)
    return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if ((d.d_query / 2) % 64 != 0 || d.d_query % 2 != 0) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (!aligned16(q) || !aligned16(keys) || !aligned16(ids) || !aligned16(weights)) return ETHOS_ERR_ALIGNMENT;
  int st;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  const int T = static_cast<int>(d.tokens);
  const int half = static_cast<int>(d.d_query / 2);
  CUtensorMap tm_q, tm_k;
  if ((st = make_tmap_bf16(&tm_q, q, d.num_heads * T, d.d_query, 128, 0, ROUTER_KB)) != ETHOS_OK) return st;
  const int box_keys = d.num_sub_keys < 256 ? static_cast<int>(d.num_sub_keys) : 256;
  if ((st = make_tmap_bf16(&tm_k, keys, 2 * d.num_sub_keys, half, box_keys, 0, ROUTER_KB)) != ETHOS_OK) return st;
  RouterGeom g;
  g.T = T;
  g.H = static_cast<int>(d.num_heads);
  g.K = static_cast<int>(d.num_sub_keys);
  g.KA = half;
  g.a_stride_h = T;
  g.a_stride_p = 0;
  g.a_col_p = half;
  g.split = 0;
  return run_score(tm_q, tm_k, g, static_cast<int>(d.top_k), ids, weights, dev_err,
                   static_cast<cudaStream_t>(stream), *dev);
}

int ethos_gemm_bf16(const void* a, const void* b, void* dptr, int64_t M, int64_t N, int64_t K, float scale,
                    int out_dtype, int* dev_err, void* stream) {
  return ethos_gemm_bf16_ex(a, K, 0, b, K, 0, dptr, N, M, N, K, scale, out_dtype, dev_err, stream);
}

int ethos_gemm_bf16_ex(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb, int b_mn_major,
                       void* dptr, int64_t ldd, int64_t M, int64_t N, int64_t K, float scale, int out_mode,
                       int* dev_err, void* stream) {
  if (!a || !b || !dptr || !dev_err) return ETHOS_ERR_INVALID_ARG;
  if (M < 1 || N < 128 || N % 128 != 0 || K < 1 || M > (int64_t(1) << 30) || K > (int64_t(1) << 30))
    return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (out_mode < 0 || out_mode > 2) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(dptr) || ldd % 8 != 0) return ETHOS_ERR_ALIGNMENT;
  int st;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GemmOperand oa{a, lda, a_mn_major != 0};
  GemmOperand ob{b, ldb, b_mn_major != 0};
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  if (out_mode == 1) {
    EpiStoreBF16 e;
    e.out = static_cast<__nv_bfloat16*>(dptr);
    e.ldo = ldd;
    e.M = m;
    e.scale = scale;
    return gemm(oa, ob, m, n, k, 1, e, dev_err, s, *dev);
  }
  if (out_mode == 2) {
    EpiAtomicF32 e;
    e.out = static_cast<float*>(dptr);
    e.ldo = ldd;
    e.M = m;
    e.scale = scale;
    return gemm(oa, ob, m, n, k, auto_ksplit(m, n, k, *dev), e, dev_err, s, *dev);
  }
  EpiStoreF32 e;
  e.out = static_cast<float*>(dptr);
  e.ldo = ldd;
  e.M = m;
  e.scale = scale;
  e.accumulate = 0;
  return gemm(oa, ob, m, n, k, 1, e, dev_err, s, *dev);
}

int ethos_test_gelu(const float* x, float* out, int64_t n, void* stream) {
  if (!x || !out || n < 2 || n % 2 != 0 || n > (int64_t(1) << 31)) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(out)) return ETHOS_ERR_ALIGNMENT;
  int st;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  const int64_t pairs = n / 2;
  int64_t blocks = (pairs + 255) / 256;
  if (blocks > 8 * dev->sm_count) blocks = 8 * dev->sm_count;
  count_launch();
  k_test_gelu<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, out, n);
  return launch_status();
}

int ethos_set_wait_limit_ns(uint64_t limit_ns) {
  if (limit_ns == 0) limit_ns = kWaitLimitNs;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ETHOS_ERR_NO_DEVICE;
  const unsigned long long v = limit_ns;
  if (cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v)) != cudaSuccess) return ETHOS_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return ETHOS_ERR_CUDA;
  return ETHOS_OK;
}

int ethos_test_gemm_withhold(const void* a, const void* b, float* dptr, int64_t M, int64_t N, int64_t K,
                             int64_t hold_unit, int* dev_err, void* stream) {
  if (!a || !b || !dptr || !dev_err || hold_unit < 0) return ETHOS_ERR_INVALID_ARG;
  if (M < 1 || N < 128 || N % 128 != 0 || K < 8 || K % 8 != 0 || M > (int64_t(1) << 30) ||
      K > (int64_t(1) << 30))
    return ETHOS_ERR_UNSUPPORTED_SHAPE;
  if (!aligned16(a) || !aligned16(b) || !aligned16(dptr)) return ETHOS_ERR_ALIGNMENT;
  int st;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  CUtensorMap ta, tb;
  if ((st = make_tmap_bf16(&ta, a, M, K, 128)) != ETHOS_OK) return st;
  if ((st = make_tmap_bf16(&tb, b, N, K, 128)) != ETHOS_OK) return st;
  EpiStoreF32 e;
  e.out = dptr;
  e.ldo = N;
  e.M = static_cast<int>(M);
  e.scale = 1.f;
  e.accumulate = 0;
  return launch_gemm_t<EpiStoreF32, false, false, 128>(ta, tb, static_cast<int>(M), static_cast<int>(N),
                                                       static_cast<int>(K), 1, e, dev_err,
                                                       static_cast<cudaStream_t>(stream), *dev,
                                                       static_cast<int>(hold_unit));
}

}  // extern "C"

namespace {
// Device address of g_noalloc_scratch for the current device, looked up on
// the first call per device (with that device current) and cached.
void* noalloc_scratch(int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = ETHOS_ERR_NO_DEVICE;
    return nullptr;
  }
  static std::mutex mu;
  static void* addr[64];
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = ETHOS_ERR_CUDA;
      return nullptr;
    }
    addr[dev] = p;
  }
  *status = ETHOS_OK;
  return addr[dev];
}
}  // namespace

extern "C" {

int ethos_router_forward_noalloc(const ethos_dims* dims, const void* x, const void* w_cat, const float* bn,
                                 float bn_eps, const void* key_cat, int32_t* ids, float* weights, int* dev_err,
                                 void* stream) {
  int st = check_dims_impl(dims);
  if (st != ETHOS_OK) return st;
  if (!x || !w_cat || !bn || !key_cat || !ids || !weights || !dev_err) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_cat) || !aligned16(bn) || !aligned16(key_cat) || !aligned16(ids) ||
      !aligned16(weights))
    return ETHOS_ERR_ALIGNMENT;
  const ethos_dims& d = *dims;
  const size_t HQ = static_cast<size_t>(d.num_heads * d.d_query);
  const size_t colp_bytes = (HQ * sizeof(float2) + 255) & ~static_cast<size_t>(255);
  const size_t qs_bytes = static_cast<size_t>(d.tokens) * HQ * 2 * sizeof(__nv_bfloat16);
  if (colp_bytes + qs_bytes > ETHOS_NOALLOC_SCRATCH_BYTES) return ETHOS_ERR_SCRATCH_LIMIT;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  char* scratch = static_cast<char*>(noalloc_scratch(&st));
  if (st != ETHOS_OK) return st;
  FwdScratch s{};
  s.colp = reinterpret_cast<float2*>(scratch);
  s.qs = reinterpret_cast<__nv_bfloat16*>(scratch + colp_bytes);
  s.slabs = 0;
  return router_core(d, x, w_cat, const_cast<float*>(bn), bn_eps, 0.f, 0, key_cat, ids, weights, false, nullptr, s,
                     s.qs, nullptr, false, nullptr, dev_err, static_cast<cudaStream_t>(stream), *dev);
}

size_t ethos_backward_workspace_size(const ethos_dims* dims) {
  if (check_dims_impl(dims) != ETHOS_OK) return 0;
  Carve c{nullptr, 0, 0};
  BwdScratch s;
  carve_backward(c, *dims, &s);
  return c.off + 256;
}

int ethos_layer_backward(const ethos_dims* dims, int bn_training, float bn_eps, const void* dy, int dy_fp32,
                         const void* x, const void* w_cat, const float* bn, const void* key_cat, const void* latents,
                         const void* w1, const void* wv, const int32_t* ids, const float* weights,
                         const float* save_xp, const void* save_hacc, const float* save_dot, const float* save_qpre,
                         const float* save_bn, const void* save_qs, const void* htab, const void* gtab,
                         void* dx, int dx_bf16, float* d_latents, float* d_w1, float* d_w2, float* d_wq,
                         float* d_bn, float* d_keys, void* workspace, size_t workspace_bytes, int* dev_err,
                         void* const* stage_events, void* stream) {
  int st = check_dims_impl(dims);
  if (st != ETHOS_OK) return st;
  if (!dy || !x || !w_cat || !bn || !key_cat || !latents || !w1 || !wv || !ids || !weights || !save_xp ||
      !save_hacc || !save_dot || !save_qpre || !save_qs || !dx || !d_latents || !d_w1 || !d_w2 || !d_wq || !d_bn ||
      !d_keys || !workspace || !dev_err)
    return ETHOS_ERR_INVALID_ARG;
  if (bn_training && !save_bn) return ETHOS_ERR_INVALID_ARG;
  if ((htab == nullptr) != (gtab == nullptr)) return ETHOS_ERR_INVALID_ARG;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  if (workspace_bytes < ethos_backward_workspace_size(dims)) return ETHOS_ERR_WORKSPACE;
  const ethos_dims& d = *dims;
  cudaStream_t sm = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<char*>(workspace), 0, workspace_bytes};
  BwdScratch s;
  carve_backward(c, d, &s);
  const int T = static_cast<int>(d.tokens), D = static_cast<int>(d.d_model);
  const int H = static_cast<int>(d.num_heads), HQ = H * static_cast<int>(d.d_query);
  const int LDU = HQ + EX_DH;
  const float invH = 1.0f / static_cast<float>(H);
  const int cb = 256;
  const int eblocks = dev->sm_count * 8;

  // outputs that are accumulated
  if (cudaMemsetAsync(d_w2, 0, sizeof(float) * 2 * D * EX_DH, sm) != cudaSuccess) return ETHOS_ERR_CUDA;

  const void* dy16 = dy;
  if (dy_fp32) {
    count_launch();
    k_f32_to_bf16<<<eblocks, cb, 0, sm>>>(static_cast<const float*>(dy), static_cast<int64_t>(T) * D, s.dy16);
    dy16 = s.dy16;
  }
  // (1) dhacc = dy @ W_v / H            [T, dh]   (W_v read in place, MN-major)
  {
    EpiStoreF32 e;
    e.out = s.dhacc;
    e.ldo = EX_DH;
    e.M = T;
    e.scale = invH;
    e.accumulate = 0;
    if ((st = gemm(GemmOperand{dy16, D, false}, GemmOperand{wv, EX_DH, true}, T, EX_DH, D, 1, e, dev_err, sm,
                   *dev)) != ETHOS_OK)
      return st;
  }
  // (2) dW_v = dy^T hacc / H  -> d_w2[d:]
  {
    EpiAtomicF32 e;
    e.out = d_w2 + static_cast<int64_t>(D) * EX_DH;
    e.ldo = EX_DH;
    e.M = D;
    e.scale = invH;
    if ((st = gemm(GemmOperand{dy16, D, true}, GemmOperand{save_hacc, EX_DH, true}, D, EX_DH, T,
                   auto_ksplit(D, EX_DH, T, *dev), e, dev_err, sm, *dev)) != ETHOS_OK)
      return st;
  }
  // (3)-(8) experts: dw, dxp (bf16 into du[:, HQ:]), d_latents, d_w1
  {
    ExpertBwdIO io;
    io.latents = latents;
    io.w1 = w1;
    io.ids = ids;
    io.weights = weights;
    io.xp = save_xp;
    io.dot = save_dot;
    io.dhacc = s.dhacc;
    io.htab = htab;
    io.gtab = gtab;
    io.dxp = s.dxp;
    io.du = s.du;
    io.ldu = LDU;
    io.du_off = HQ;
    io.dw = s.dw;
    io.d_latents = d_latents;
    io.d_w1 = d_w1;
    if ((st = expert_bwd_core(d, io, s, dev_err, sm, *dev)) != ETHOS_OK) return st;
  }
  mark(stage_events, ETHOS_BWD_STAGE_EXPERTS, sm);  // d_latents, d_w1 final
  // (9)-(11) router: dq (bf16 into du[:, :HQ]), d_keys, d_bn
  {
    RouterBwdIO io;
    io.bn_training = bn_training;
    io.bn_eps = bn_eps;
    io.bn = bn;
    io.key_cat = key_cat;
    io.ids = ids;
    io.weights = weights;
    io.dw = s.dw;
    io.qpre = save_qpre;
    io.save_bn = save_bn;
    io.qs = save_qs;
    io.du = s.du;
    io.ldu = LDU;
    io.d_bn = d_bn;
    io.d_keys = d_keys;
    if ((st = router_bwd_core(d, io, s, dev_err, sm, *dev)) != ETHOS_OK) return st;
  }
  // (12) dx = du @ W_cat          (W_cat read in place, MN-major), in fp32 or
  // straight into bf16
  if (dx_bf16) {
    EpiStoreBF16 e;
    e.out = static_cast<__nv_bfloat16*>(dx);
    e.ldo = D;
    e.M = T;
    e.scale = 1.0f;
    if ((st = gemm(GemmOperand{s.du, LDU, false}, GemmOperand{w_cat, D, true}, T, D, LDU, 1, e, dev_err, sm,
                   *dev)) != ETHOS_OK)
      return st;
  } else {
    EpiStoreF32 e;
    e.out = static_cast<float*>(dx);
    e.ldo = D;
    e.M = T;
    e.scale = 1.0f;
    e.accumulate = 0;
    if ((st = gemm(GemmOperand{s.du, LDU, false}, GemmOperand{w_cat, D, true}, T, D, LDU, 1, e, dev_err, sm,
                   *dev)) != ETHOS_OK)
      return st;
  }
  // (13) dWq = dq^T x   [HQ, d]
  {
    EpiStoreF32 e;
    e.out = d_wq;
    e.ldo = D;
    e.M = HQ;
    e.scale = 1.0f;
    e.accumulate = 0;
    if ((st = gemm(GemmOperand{s.du, LDU, true}, GemmOperand{x, D, true}, HQ, D, T, 1, e, dev_err, sm, *dev)) !=
        ETHOS_OK)
      return st;
  }
  // (14) dW_u = x^T dxp -> d_w2[:d]   [d, dh]: 8 output tiles, so split K
  // (the tokens) over the GPU and reduce into the zeroed d_w2 with atomics
  {
    EpiAtomicF32 e;
    e.out = d_w2;
    e.ldo = EX_DH;
    e.M = D;
    e.scale = 1.0f;
    if ((st = gemm(GemmOperand{x, D, true}, GemmOperand{s.du + HQ, LDU, true}, D, EX_DH, T,
                   auto_ksplit(D, EX_DH, T, *dev), e, dev_err, sm, *dev)) != ETHOS_OK)
      return st;
  }
  mark(stage_events, ETHOS_BWD_STAGE_END, sm);
  return ETHOS_OK;
}

size_t ethos_expert_backward_workspace_size(const ethos_dims* dims) {
  if (check_dims_impl(dims) != ETHOS_OK) return 0;
  Carve c{nullptr, 0, 0};
  BwdScratch s;
  carve_expert_backward(c, *dims, &s);
  return c.off + 256;
}

int ethos_expert_backward(const ethos_dims* dims, const void* latents, const void* w1, const int32_t* ids,
                          const float* weights, const float* xp, const float* dot, const float* dhacc,
                          const void* htab, const void* gtab, float* dxp, float* d_weights, float* d_latents,
                          float* d_w1, void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
  int st = check_dims_impl(dims);
  if (st != ETHOS_OK) return st;
  if (!latents || !w1 || !ids || !weights || !xp || !dot || !dhacc || !dxp || !d_weights || !d_latents || !d_w1 ||
      !workspace || !dev_err)
    return ETHOS_ERR_INVALID_ARG;
  if ((htab == nullptr) != (gtab == nullptr)) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(xp) || !aligned16(dhacc) || !aligned16(dxp) || !aligned16(latents) || !aligned16(w1))
    return ETHOS_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  if (workspace_bytes < ethos_expert_backward_workspace_size(dims)) return ETHOS_ERR_WORKSPACE;
  const ethos_dims& d = *dims;
  Carve c{static_cast<char*>(workspace), 0, workspace_bytes};
  BwdScratch s;
  carve_expert_backward(c, d, &s);
  ExpertBwdIO io;
  io.latents = latents;
  io.w1 = w1;
  io.ids = ids;
  io.weights = weights;
  io.xp = xp;
  io.dot = dot;
  io.dhacc = dhacc;
  io.htab = htab;
  io.gtab = gtab;
  io.dxp = dxp;
  io.du = s.du;
  io.ldu = EX_DH;
  io.du_off = 0;
  io.dw = d_weights;
  io.d_latents = d_latents;
  io.d_w1 = d_w1;
  return expert_bwd_core(d, io, s, dev_err, static_cast<cudaStream_t>(stream), *dev);
}

size_t ethos_router_backward_workspace_size(const ethos_dims* dims) {
  if (check_dims_impl(dims) != ETHOS_OK) return 0;
  Carve c{nullptr, 0, 0};
  BwdScratch s;
  RouterBwdExtra x;
  carve_router_backward(c, *dims, &s, &x);
  return c.off + 256;
}

int ethos_router_backward(const ethos_dims* dims, int bn_training, float bn_eps, const void* x, const void* w_cat,
                          const float* bn, const void* key_cat, const int32_t* ids, const float* weights,
                          const float* d_weights, const float* save_qpre, const float* save_bn, float* dx,
                          int accumulate_dx, float* d_wq, float* d_bn, float* d_keys, void* workspace,
                          size_t workspace_bytes, int* dev_err, void* stream) {
  int st = check_dims_impl(dims);
  if (st != ETHOS_OK) return st;
  if (!x || !w_cat || !bn || !key_cat || !ids || !weights || !d_weights || !save_qpre || !dx || !d_wq || !d_bn ||
      !d_keys || !workspace || !dev_err)
    return ETHOS_ERR_INVALID_ARG;
  if (bn_training && !save_bn) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_cat) || !aligned16(save_qpre) || !aligned16(dx) || !aligned16(d_wq) ||
      !aligned16(key_cat))
    return ETHOS_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  if (workspace_bytes < ethos_router_backward_workspace_size(dims)) return ETHOS_ERR_WORKSPACE;
  const ethos_dims& d = *dims;
  cudaStream_t sm = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<char*>(workspace), 0, workspace_bytes};
  BwdScratch s;
  RouterBwdExtra xs;
  carve_router_backward(c, d, &s, &xs);
  const int T = static_cast<int>(d.tokens), D = static_cast<int>(d.d_model);
  const int H = static_cast<int>(d.num_heads), dq = static_cast<int>(d.d_query), HQ = H * dq;
  const int cb = 256;
  // the forward's normalised queries, recomputed from qpre with the affine
  // the forward used (batch statistics or running statistics)
  count_launch();
  if (bn_training)
    k_bn_colp_from_stats<<<(HQ + cb - 1) / cb, cb, 0, sm>>>(bn, save_bn, HQ, xs.colp);
  else
    k_bn_eval_colp<<<(HQ + cb - 1) / cb, cb, 0, sm>>>(bn, HQ, bn_eps, 1, xs.colp);
  count_launch();
  k_bn_apply<<<bn_rows_grid(HQ, T, cb, *dev), cb, 0, sm>>>(save_qpre, xs.colp, T, H, dq, xs.qs);
  if ((st = launch_status()) != ETHOS_OK) return st;
  RouterBwdIO io;
  io.bn_training = bn_training;
  io.bn_eps = bn_eps;
  io.bn = bn;
  io.key_cat = key_cat;
  io.ids = ids;
  io.weights = weights;
  io.dw = d_weights;
  io.qpre = save_qpre;
  io.save_bn = save_bn;
  io.qs = xs.qs;
  io.du = s.du;
  io.ldu = HQ;
  io.d_bn = d_bn;
  io.d_keys = d_keys;
  if ((st = router_bwd_core(d, io, s, dev_err, sm, *dev)) != ETHOS_OK) return st;
  // dx (+)= dq @ W_q    (W_q = the first H*dq rows of w_cat, read in place)
  {
    EpiStoreF32 e;
    e.out = dx;
    e.ldo = D;
    e.M = T;
    e.scale = 1.0f;
    e.accumulate = accumulate_dx ? 1 : 0;
    if ((st = gemm(GemmOperand{s.du, HQ, false}, GemmOperand{w_cat, D, true}, T, D, HQ, 1, e, dev_err, sm,
                   *dev)) != ETHOS_OK)
      return st;
  }
  // dWq = dq^T x   [HQ, d]
  {
    EpiStoreF32 e;
    e.out = d_wq;
    e.ldo = D;
    e.M = HQ;
    e.scale = 1.0f;
    e.accumulate = 0;
    if ((st = gemm(GemmOperand{s.du, HQ, true}, GemmOperand{x, D, true}, HQ, D, T, 1, e, dev_err, sm, *dev)) !=
        ETHOS_OK)
      return st;
  }
  return ETHOS_OK;
}

int ethos_adamw_step(const ethos_adam_tensor* tensors, int num_tensors, int64_t max_n, float lr, float beta1,
                     float beta2, float eps, float weight_decay, int64_t step, const float* grad_scale, int* dev_err,
                     void* stream) {
  (void)dev_err;
  if (num_tensors == 0 || max_n == 0) return ETHOS_OK;
  if (tensors == nullptr || num_tensors < 0 || num_tensors > 65535 || max_n < 0 || step < 1)
    return ETHOS_ERR_INVALID_ARG;
  if (!(beta1 >= 0.f && beta1 < 1.f && beta2 >= 0.f && beta2 < 1.f && eps > 0.f)) return ETHOS_ERR_INVALID_ARG;
  int st;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  AdamScalars s;
  s.lr = lr;
  s.beta1 = beta1;
  s.beta2 = beta2;
  s.eps = eps;
  s.wd = weight_decay;
  s.step_size = static_cast<float>(lr / (1.0 - std::pow(static_cast<double>(beta1), static_cast<double>(step))));
  s.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(static_cast<double>(beta2), static_cast<double>(step))));
  const int threads = 256;
  int64_t bx = (max_n + threads * 4 - 1) / (threads * 4);
  const int64_t cap = static_cast<int64_t>(dev->sm_count) * 8;
  if (bx > cap) bx = cap;
  if (bx < 1) bx = 1;
  count_launch();
  k_adamw<<<dim3(static_cast<unsigned>(bx), static_cast<unsigned>(num_tensors)), threads, 0,
            static_cast<cudaStream_t>(stream)>>>(tensors, s, grad_scale);
  return launch_status();
}

size_t ethos_grad_clip_workspace_size(void) { return sizeof(double) * GRAD_CLIP_BLOCKS; }

int ethos_grad_clip_coef(const ethos_adam_tensor* tensors, int num_tensors, float max_norm, void* workspace,
                         size_t workspace_bytes, float* out, int* dev_err, void* stream) {
  (void)dev_err;
  if (tensors == nullptr || out == nullptr || num_tensors <= 0 || !(max_norm > 0.f)) return ETHOS_ERR_INVALID_ARG;
  if (workspace == nullptr || workspace_bytes < ethos_grad_clip_workspace_size() ||
      (reinterpret_cast<uintptr_t>(workspace) & 7u) != 0)
    return ETHOS_ERR_WORKSPACE;
  int st;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  const cudaStream_t sm = static_cast<cudaStream_t>(stream);
  double* partial = static_cast<double*>(workspace);
  count_launch();
  k_grad_sqnorm<<<GRAD_CLIP_BLOCKS, GRAD_CLIP_THREADS, 0, sm>>>(tensors, num_tensors, partial);
  if ((st = launch_status()) != ETHOS_OK) return st;
  count_launch();
  k_grad_clip_coef<<<1, GRAD_CLIP_THREADS, 0, sm>>>(partial, GRAD_CLIP_BLOCKS, max_norm, out);
  return launch_status();
}

}  // extern "C"

// ===================================================== fp32 arithmetic path --
namespace {

// Extra shape rules of the fp32 path: its score GEMMs need d_query / 2 to be
// a multiple of 128 (their N tile), and the padded key count Kp below.
int check_dims_f32(const ethos_dims* d) {
  const int st = check_dims_impl(d);
  if (st != ETHOS_OK) return st;
  if ((d->d_query / 2) % 128 != 0) return ETHOS_ERR_UNSUPPORTED_SHAPE;
  return ETHOS_OK;
}

// Sub-key count rounded up to the GEMM's 128-column N tile (score rows are
// Kp wide; the extra key rows are zero and never selected).
int64_t padded_keys(const ethos_dims& d) { return (d.num_sub_keys + 127) / 128 * 128; }

// Split an fp32 [rows, cols] matrix (row pitch lds) into bf16 segments (see
// k_split_bf16).
int launch_split(const float* src, int64_t rows, int cols, int64_t lds, __nv_bfloat16* dst, int64_t ldd,
                 int64_t seg_off, int nseg, int parts, cudaStream_t stream, const DeviceInfo& dev) {
  const int tx = 128;
  const int gx = (cols + tx - 1) / tx;
  int64_t gy = (static_cast<int64_t>(dev.sm_count) * 16) / gx;
  if (gy < 1) gy = 1;
  if (gy > rows) gy = rows;
  if (gy > 65535) gy = 65535;
  count_launch();
  k_split_bf16<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), tx, 0, stream>>>(
      src, rows, cols, lds, dst, ldd, seg_off, nseg, parts);
  return launch_status();
}

// Separate hi / lo arrays of an fp32 [rows, cols] matrix: dst holds hi
// [rows][cols] then lo [rows][cols].
int split2(const float* src, int64_t rows, int cols, int64_t lds, __nv_bfloat16* dst, cudaStream_t stream,
           const DeviceInfo& dev) {
  return launch_split(src, rows, cols, lds, dst, cols, rows * cols, 2, SPLIT_HI_LO, stream, dev);
}

// The K-concatenated operands of the six-product projection GEMM, row-major
// [rows][6 * cols]: A = [hi | r | lo | lo | hi | hi], B = [r | hi | lo | hi |
// lo | hi] (hi*hi last; see SPLIT6_A).
int split6(const float* src, int64_t rows, int cols, int64_t lds, __nv_bfloat16* dst, bool as_b,
           cudaStream_t stream, const DeviceInfo& dev) {
  return launch_split(src, rows, cols, lds, dst, 6 * static_cast<int64_t>(cols), cols, 6,
                      as_b ? SPLIT6_B : SPLIT6_A, stream, dev);
}

// A split operand: hi and lo bf16 arrays of one layout (row pitch ld,
// K-major or MN-major as in GemmOperand).
struct SplitOperand {
  const __nv_bfloat16* hi;
  const __nv_bfloat16* lo;
  int64_t ld;
  bool mn_major;
};

// D (=|+=) scale * A B^T in fp32 from split operands: hi*hi, then lo*hi and
// hi*lo accumulated.  atomic: all three reduce into D with fp32 atomics
// (split-K allowed; D pre-initialised by the caller); else the first stores
// and the other two add.
int gemm_split(const SplitOperand& a, const SplitOperand& b, int M, int N, int K, float* out, int64_t ldo,
               float scale, bool atomic, int* err, cudaStream_t stream, const DeviceInfo& dev) {
  const GemmOperand A[3] = {{a.hi, a.ld, a.mn_major}, {a.lo, a.ld, a.mn_major}, {a.hi, a.ld, a.mn_major}};
  const GemmOperand B[3] = {{b.hi, b.ld, b.mn_major}, {b.hi, b.ld, b.mn_major}, {b.lo, b.ld, b.mn_major}};
  const int ks = atomic ? auto_ksplit(M, N, K, dev) : 1;
  for (int i = 0; i < 3; ++i) {
    int st;
    if (atomic) {
      EpiAtomicF32 e;
      e.out = out;
      e.ldo = ldo;
      e.M = M;
      e.scale = scale;
      st = gemm(A[i], B[i], M, N, K, ks, e, err, stream, dev);
    } else {
      EpiStoreF32 e;
      e.out = out;
      e.ldo = ldo;
      e.M = M;
      e.scale = scale;
      e.accumulate = i > 0 ? 1 : 0;
      st = gemm(A[i], B[i], M, N, K, 1, e, err, stream, dev);
    }
    if (st != ETHOS_OK) return st;
  }
  return ETHOS_OK;
}

dim3 rows_grid(int cols, int64_t rows, int threads, const DeviceInfo& dev) {
  const int gx = (cols + threads - 1) / threads;
  int64_t gy = static_cast<int64_t>(dev.sm_count) * 8 / gx;
  if (gy < 1) gy = 1;
  if (gy > rows) gy = rows;
  if (gy > 65535) gy = 65535;
  return dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
}

int warp_blocks(int64_t items, const DeviceInfo& dev) {
  int64_t b = (items + 7) / 8;  // 8 warps per 256-thread block
  const int64_t cap = static_cast<int64_t>(dev.sm_count) * 16;
  if (b > cap) b = cap;
  return b < 1 ? 1 : static_cast<int>(b);
}

struct Fwd32Scratch {
  __nv_bfloat16* x6;      // [T][6d]
  __nv_bfloat16* w6;      // [ncat][6d]
  float* pcat;            // [T][ncat] projection partial over K [0, 5.5d)
  float* qpre;            // [T][HQ]
  float* xp;              // [T][dh]
  float2* colp;           // [HQ]
  float* save_bn;         // [2][HQ]
  float* bn_part;
  float* qhat;            // [2][H][T][half]
  __nv_bfloat16* qhat_s;  // hi, lo of qhat
  __nv_bfloat16* keys_s;  // hi [2][Kp][half], lo [2][Kp][half]
  float* scores;          // [2][H*T][Kp]
  __nv_bfloat16* e_s;     // hi, lo [N][dl]
  __nv_bfloat16* w1_s;    // hi, lo [dh][dl]
  float* tab;             // [N][dh]
  float* hacc;            // [T][dh]
  __nv_bfloat16* hacc_s;  // hi, lo [T][dh]
  __nv_bfloat16* wv_s;    // hi, lo [d][dh]
  float* dot;             // [T][R]
  int slabs;
};

// Scratch of the fp32 forward; a `have_*` flag means the caller passes that
// buffer (save outputs), so no scratch is carved for it.
void carve_forward_f32(Carve& c, const ethos_dims& d, int bn_training, bool experts, bool have_qpre, bool have_xp,
                       bool have_bn, bool have_qhat, bool have_tab, bool have_hacc, bool have_dot, Fwd32Scratch* s) {
  const int64_t T = d.tokens, D = d.d_model, H = d.num_heads, HQ = H * d.d_query, half = d.d_query / 2;
  const int64_t dh = d.d_hidden, N = d.num_experts, Kp = padded_keys(d), R = H * d.top_k;
  const int64_t ncat = experts ? HQ + dh : HQ;
  s->x6 = c.take<__nv_bfloat16>(static_cast<size_t>(T * 6 * D));
  s->w6 = c.take<__nv_bfloat16>(static_cast<size_t>(ncat * 6 * D));
  s->pcat = c.take<float>(static_cast<size_t>(T * ncat));
  s->qpre = have_qpre ? nullptr : c.take<float>(static_cast<size_t>(T * HQ));
  s->xp = (!experts || have_xp) ? nullptr : c.take<float>(static_cast<size_t>(T * dh));
  s->colp = c.take<float2>(static_cast<size_t>(HQ));
  s->slabs = static_cast<int>((T + BN_ROWS_PER_SLAB - 1) / BN_ROWS_PER_SLAB);
  s->save_bn = (bn_training && !have_bn) ? c.take<float>(static_cast<size_t>(2 * HQ)) : nullptr;
  s->bn_part = bn_training ? c.take<float>(static_cast<size_t>(s->slabs) * HQ * 2) : nullptr;
  s->qhat = have_qhat ? nullptr : c.take<float>(static_cast<size_t>(2 * H * T * half));
  s->qhat_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * 2 * H * T * half));
  s->keys_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * 2 * Kp * half));
  s->scores = c.take<float>(static_cast<size_t>(2 * H * T * Kp));
  if (experts) {
    s->e_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * N * d.d_latent));
    s->w1_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * dh * d.d_latent));
    s->tab = have_tab ? nullptr : c.take<float>(static_cast<size_t>(N * dh));
    s->hacc = have_hacc ? nullptr : c.take<float>(static_cast<size_t>(T * dh));
    s->hacc_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * T * dh));
    s->wv_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * D * dh));
    s->dot = have_dot ? nullptr : c.take<float>(static_cast<size_t>(T * R));
  } else {
    s->e_s = s->w1_s = s->hacc_s = s->wv_s = nullptr;
    s->tab = s->hacc = s->dot = nullptr;
  }
}

// Pre-activations of the expert table in fp32 (E @ W1^T on split operands),
// then GELU in place (and its derivative into g when given).
int build_table_f32(const ethos_dims& d, const float* latents, const float* w1, __nv_bfloat16* e_s,
                    __nv_bfloat16* w1_s, float* tab, float* g, int* err, cudaStream_t stream, const DeviceInfo& dev) {
  const int64_t N = d.num_experts, dl = d.d_latent, dh = d.d_hidden;
  int st;
  if ((st = split2(latents, N, static_cast<int>(dl), dl, e_s, stream, dev)) != ETHOS_OK) return st;
  if ((st = split2(w1, dh, static_cast<int>(dl), dl, w1_s, stream, dev)) != ETHOS_OK) return st;
  const SplitOperand a{e_s, e_s + N * dl, dl, false};
  const SplitOperand b{w1_s, w1_s + dh * dl, dl, false};
  if ((st = gemm_split(a, b, static_cast<int>(N), static_cast<int>(dh), static_cast<int>(dl), tab, dh, 1.0f, false,
                       err, stream, dev)) != ETHOS_OK)
    return st;
  const int64_t n = N * dh;
  int64_t blocks = (n / 2 + 255) / 256;
  if (blocks > dev.sm_count * 16) blocks = dev.sm_count * 16;
  count_launch();
  k_gelu_table_f32<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(tab, g, n);
  return launch_status();
}

struct Bwd32Scratch {
  __nv_bfloat16* dy_s;    // hi, lo [T][d]
  __nv_bfloat16* wv_s;    // hi, lo [d][dh]
  float* dhacc;           // [T][dh]
  __nv_bfloat16* hacc_s;  // hi, lo [T][dh]
  __nv_bfloat16* e_s;     // hi, lo [N][dl]
  __nv_bfloat16* w1_s;    // hi, lo [dh][dl]
  float* tab;             // [N][dh] (when the forward kept none)
  float* gtab;            // [N][dh]
  float* dw;              // [T][R]
  float* ca;
  float* cd;
  float* du;              // [T][LDU] = [dq | dxp]
  __nv_bfloat16* du_s;    // hi, lo [T][LDU]
  int* cnt;
  int* offs;
  int* cursor;
  int* bsums;
  int* total;
  int* perm;
  float* dP;              // [N][dh]
  __nv_bfloat16* dP_s;    // hi, lo
  float* dqhat;           // [T][HQ]
  float* dS;              // [2][H*T][K]
  __nv_bfloat16* dS_s;    // hi, lo
  __nv_bfloat16* qhat_s;  // hi, lo [2][H*T][half]
  float* part;
  float* coef;
  float* stats;
  __nv_bfloat16* wcat_s;  // hi, lo [ncat][d]
  __nv_bfloat16* x_s;     // hi, lo [T][d]
  int slabs;
};

void carve_backward_f32(Carve& c, const ethos_dims& d, bool have_tables, Bwd32Scratch* s) {
  const int64_t T = d.tokens, D = d.d_model, H = d.num_heads, HQ = H * d.d_query, half = d.d_query / 2;
  const int64_t dh = d.d_hidden, dl = d.d_latent, N = d.num_experts, K = d.num_sub_keys, R = H * d.top_k;
  const int64_t LDU = HQ + dh;
  s->dy_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * T * D));
  s->wv_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * D * dh));
  s->dhacc = c.take<float>(static_cast<size_t>(T * dh));
  s->hacc_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * T * dh));
  s->e_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * N * dl));
  s->w1_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * dh * dl));
  s->tab = have_tables ? nullptr : c.take<float>(static_cast<size_t>(N * dh));
  s->gtab = have_tables ? nullptr : c.take<float>(static_cast<size_t>(N * dh));
  s->dw = c.take<float>(static_cast<size_t>(T * R));
  s->ca = c.take<float>(static_cast<size_t>(T * R));
  s->cd = c.take<float>(static_cast<size_t>(T * R));
  s->du = c.take<float>(static_cast<size_t>(T * LDU));
  s->du_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * T * LDU));
  s->cnt = c.take<int>(static_cast<size_t>(N));
  s->offs = c.take<int>(static_cast<size_t>(N));
  s->cursor = c.take<int>(static_cast<size_t>(N));
  s->bsums = c.take<int>(1024);
  s->total = c.take<int>(1);
  s->perm = c.take<int>(static_cast<size_t>(T * R));
  s->dP = c.take<float>(static_cast<size_t>(N * dh));
  s->dP_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * N * dh));
  s->dqhat = c.take<float>(static_cast<size_t>(T * HQ));
  s->dS = c.take<float>(static_cast<size_t>(2 * H * T * K));
  s->dS_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * 2 * H * T * K));
  s->qhat_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * 2 * H * T * half));
  s->slabs = static_cast<int>((T + BN_ROWS_PER_SLAB - 1) / BN_ROWS_PER_SLAB);
  s->part = c.take<float>(static_cast<size_t>(s->slabs) * HQ * 2);
  s->coef = c.take<float>(static_cast<size_t>(4 * HQ));
  s->stats = c.take<float>(static_cast<size_t>(2 * HQ));
  s->wcat_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * LDU * D));
  s->x_s = c.take<__nv_bfloat16>(static_cast<size_t>(2 * T * D));
}

template <int TOPK>
int launch_topk_f32(const float* scores, int64_t ldk, const ethos_dims& d, int32_t* ids, float* w,
                    cudaStream_t stream, const DeviceInfo& dev) {
  count_launch();
  k_topk_f32<TOPK><<<warp_blocks(d.num_heads * d.tokens, dev), 256, 0, stream>>>(
      scores, ldk, static_cast<int>(d.tokens), static_cast<int>(d.num_heads), static_cast<int>(d.num_sub_keys), ids,
      w);
  return launch_status();
}

template <int TOPK>
int launch_router_bwd_f32(const ethos_dims& d, const int32_t* ids, const float* w, const float* dw,
                          const float* keys, float* dqhat, float* dS, cudaStream_t stream, const DeviceInfo& dev) {
  count_launch();
  k_router_bwd_f32<TOPK><<<warp_blocks(d.num_heads * d.tokens, dev), 256, 0, stream>>>(
      ids, w, dw, keys, dqhat, dS, static_cast<int>(d.tokens), static_cast<int>(d.num_heads),
      static_cast<int>(d.num_sub_keys), static_cast<int>(d.d_query));
  return launch_status();
}

}  // namespace

extern "C" {

size_t ethos_forward_workspace_size_f32(const ethos_dims* dims, int bn_training) {
  if (check_dims_f32(dims) != ETHOS_OK) return 0;
  Carve c{nullptr, 0, 0};
  Fwd32Scratch s;
  carve_forward_f32(c, *dims, bn_training, true, false, false, false, false, false, false, false, &s);
  return c.off + 256;
}

int ethos_layer_forward_f32(const ethos_dims* dims, const float* x, const float* w_cat, float* bn, float bn_eps,
                            float bn_momentum, int bn_training, const float* keys, const float* latents,
                            const float* w1, const float* wv, float* y, int32_t* ids, float* weights,
                            float* save_xp, float* save_hacc, float* save_dot, float* save_qpre, float* save_bn,
                            float* save_qhat, float* save_htab, float* save_gtab, void* workspace,
                            size_t workspace_bytes, int* dev_err, void* stream) {
  int st = check_dims_f32(dims);
  if (st != ETHOS_OK) return st;
  const bool experts = y != nullptr;
  if (!x || !w_cat || !bn || !keys || !ids || !weights || !workspace || !dev_err) return ETHOS_ERR_INVALID_ARG;
  if (experts && (!latents || !w1 || !wv)) return ETHOS_ERR_INVALID_ARG;
  if (save_gtab != nullptr && save_htab == nullptr) return ETHOS_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_cat) || !aligned16(keys) || (experts && (!aligned16(latents) ||
      !aligned16(w1) || !aligned16(wv) || !aligned16(y))))
    return ETHOS_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  const ethos_dims& d = *dims;
  Carve c{static_cast<char*>(workspace), 0, workspace_bytes};
  Fwd32Scratch s;
  carve_forward_f32(c, d, bn_training, experts, save_qpre != nullptr, save_xp != nullptr, save_bn != nullptr,
                    save_qhat != nullptr, save_htab != nullptr, save_hacc != nullptr, save_dot != nullptr, &s);
  if (c.off > workspace_bytes) return ETHOS_ERR_WORKSPACE;
  cudaStream_t sm = static_cast<cudaStream_t>(stream);
  const int T = static_cast<int>(d.tokens), D = static_cast<int>(d.d_model), H = static_cast<int>(d.num_heads);
  const int dq = static_cast<int>(d.d_query), HQ = H * dq, half = dq / 2, dh = static_cast<int>(d.d_hidden);
  const int K = static_cast<int>(d.num_sub_keys), R = H * static_cast<int>(d.top_k);
  const int N = static_cast<int>(d.num_experts);
  const int64_t Kp = padded_keys(d), HT = static_cast<int64_t>(H) * T;
  const int ncat = experts ? HQ + dh : HQ;
  float* qpre = save_qpre ? save_qpre : s.qpre;
  float* xp = experts ? (save_xp ? save_xp : s.xp) : nullptr;
  float* sbn = save_bn ? save_bn : s.save_bn;
  float* qhat = save_qhat ? save_qhat : s.qhat;
  const int cb = 256;

  // (1) queries and x_proj on the six-product K-concatenated split operands
  //     (fp32-level qpre, which small-batch BatchNorm amplifies), the bias
  //     added in the epilogue (model.py:215, 326).  Two launches, each
  //     accumulating from zero in TMEM: the small products and the first half
  //     of hi*hi into pcat, then the second half of hi*hi, which adds pcat in
  //     its epilogue.  Each accumulation chain is then D / 32 steps of the
  //     large products long instead of D / 16.
  if ((st = split6(x, T, D, D, s.x6, false, sm, *dev)) != ETHOS_OK) return st;
  if ((st = split6(w_cat, ncat, D, D, s.w6, true, sm, *dev)) != ETHOS_OK) return st;
  if (!bn_training) {
    count_launch();
    k_bn_eval_colp<<<(HQ + cb - 1) / cb, cb, 0, sm>>>(bn, HQ, bn_eps, 1, s.colp);
  }
  {
    const int k0 = 5 * D + D / 2;  // d_model % 256 == 0: both slices 16-byte aligned, K % 64 == 0
    EpiStoreF32 ep;
    ep.out = s.pcat;
    ep.ldo = ncat;
    ep.M = T;
    ep.scale = 1.0f;
    ep.accumulate = 0;
    if ((st = gemm(GemmOperand{s.x6, 6 * D, false}, GemmOperand{s.w6, 6 * D, false}, T, ncat, k0, 1, ep, dev_err,
                   sm, *dev)) != ETHOS_OK)
      return st;
    CUtensorMap tm_x, tm_w;
    if ((st = make_tmap_bf16(&tm_x, s.x6 + k0, T, D / 2, 128, 6 * D)) != ETHOS_OK) return st;
    if ((st = make_tmap_bf16(&tm_w, s.w6 + k0, ncat, D / 2, G2_BN / 2, 6 * D)) != ETHOS_OK) return st;
    EpiProj epi;
    epi.M = T;
    epi.HQ = HQ;
    epi.dq = dq;
    epi.dh = dh;
    epi.mode = 1;
    epi.bias = bn;
    epi.colp = s.colp;
    epi.qs = nullptr;
    epi.qpre = qpre;
    epi.xp = xp;
    epi.part = s.pcat;
    epi.ldp = ncat;
    if ((st = launch_gemm2sm(tm_x, tm_w, T, ncat, D / 2, epi, dev_err, sm, *dev)) != ETHOS_OK) return st;
  }
  // (2) BatchNorm (model.py:216): batch statistics and running-stat update in
  //     training mode, running statistics in eval mode
  if (bn_training) {
    dim3 grid_p((HQ + cb - 1) / cb, s.slabs);
    count_launch();
    k_bn_partial<<<grid_p, cb, 0, sm>>>(qpre, T, HQ, s.bn_part);
    count_launch();
    k_bn_finalize<<<(HQ + cb - 1) / cb, cb, 0, sm>>>(qpre, s.bn_part, T, HQ, s.slabs, bn + HQ, bn + 2 * HQ,
                                                     bn + 3 * HQ, bn + 4 * HQ, bn_eps, bn_momentum, sbn, s.colp);
  }
  count_launch();
  k_bn_apply_f32<<<rows_grid(HQ, T, cb, *dev), cb, 0, sm>>>(qpre, s.colp, bn_training ? sbn : bn + 3 * HQ,
                                                            bn + 2 * HQ, T, H, dq, qhat);
  if ((st = launch_status()) != ETHOS_OK) return st;
  // (3) sub-key scores of both halves (model.py:217-221), then top-k, grid
  //     top-k, softmax and id decode (model.py:224-245)
  if ((st = split2(qhat, 2 * HT, half, half, s.qhat_s, sm, *dev)) != ETHOS_OK) return st;
  if (cudaMemsetAsync(s.keys_s, 0, sizeof(__nv_bfloat16) * 2 * 2 * Kp * half, sm) != cudaSuccess)
    return ETHOS_ERR_CUDA;
  for (int p = 0; p < 2; ++p) {
    st = launch_split(keys + static_cast<int64_t>(p) * K * half, K, half, half,
                      s.keys_s + static_cast<int64_t>(p) * Kp * half, half, 2 * Kp * half, 2, SPLIT_HI_LO, sm, *dev);
    if (st != ETHOS_OK) return st;
  }
  const int64_t qlo = 2 * HT * half;
  for (int p = 0; p < 2; ++p) {
    const SplitOperand a{s.qhat_s + p * HT * half, s.qhat_s + qlo + p * HT * half, half, false};
    const SplitOperand b{s.keys_s + p * Kp * half, s.keys_s + 2 * Kp * half + p * Kp * half, half, false};
    if ((st = gemm_split(a, b, static_cast<int>(HT), static_cast<int>(Kp), half, s.scores + p * HT * Kp, Kp, 1.0f,
                         false, dev_err, sm, *dev)) != ETHOS_OK)
      return st;
  }
  switch (d.top_k) {
    case 4: st = launch_topk_f32<4>(s.scores, Kp, d, ids, weights, sm, *dev); break;
    case 8: st = launch_topk_f32<8>(s.scores, Kp, d, ids, weights, sm, *dev); break;
    default: st = launch_topk_f32<16>(s.scores, Kp, d, ids, weights, sm, *dev); break;
  }
  if (st != ETHOS_OK || !experts) return st;
  // (4) expert table H = gelu(E W1^T) in fp32, once per expert (model.py:323)
  float* tab = save_htab ? save_htab : s.tab;
  if ((st = build_table_f32(d, latents, w1, s.e_s, s.w1_s, tab, save_gtab, dev_err, sm, *dev)) != ETHOS_OK)
    return st;
  // (5) per token: dot, activation, weighted hidden sum (model.py:320-338)
  float* hacc = save_hacc ? save_hacc : s.hacc;
  float* dot = save_dot ? save_dot : s.dot;
  count_launch();
  k_gather_f32<<<warp_blocks(T, *dev), 256, 0, sm>>>(tab, ids, weights, xp, hacc, dot, T, R, N, dev_err);
  if ((st = launch_status()) != ETHOS_OK) return st;
  // (6) y = hacc W_v^T / H (model.py:332-341)
  if ((st = split2(hacc, T, dh, dh, s.hacc_s, sm, *dev)) != ETHOS_OK) return st;
  if ((st = split2(wv, D, dh, dh, s.wv_s, sm, *dev)) != ETHOS_OK) return st;
  const SplitOperand a{s.hacc_s, s.hacc_s + static_cast<int64_t>(T) * dh, dh, false};
  const SplitOperand b{s.wv_s, s.wv_s + static_cast<int64_t>(D) * dh, dh, false};
  return gemm_split(a, b, T, D, dh, y, D, 1.0f / static_cast<float>(H), false, dev_err, sm, *dev);
}

size_t ethos_backward_workspace_size_f32(const ethos_dims* dims) {
  if (check_dims_f32(dims) != ETHOS_OK) return 0;
  Carve c{nullptr, 0, 0};
  Bwd32Scratch s;
  carve_backward_f32(c, *dims, false, &s);
  return c.off + 256;
}

int ethos_layer_backward_f32(const ethos_dims* dims, int bn_training, float bn_eps, const float* dy, const float* x,
                             const float* w_cat, const float* bn, const float* keys, const float* latents,
                             const float* w1, const float* wv, const int32_t* ids, const float* weights,
                             const float* save_xp, const float* save_hacc, const float* save_dot,
                             const float* save_qpre, const float* save_bn, const float* save_qhat, const float* htab,
                             const float* gtab, float* dx, float* d_latents, float* d_w1, float* d_w2, float* d_wq,
                             float* d_bn, float* d_keys, void* workspace, size_t workspace_bytes, int* dev_err,
                             void* const* stage_events, void* stream) {
  int st = check_dims_f32(dims);
  if (st != ETHOS_OK) return st;
  if (!dy || !x || !w_cat || !bn || !keys || !latents || !w1 || !wv || !ids || !weights || !save_xp ||
      !save_hacc || !save_dot || !save_qpre || !save_qhat || !dx || !d_latents || !d_w1 || !d_w2 || !d_wq ||
      !d_bn || !d_keys || !workspace || !dev_err)
    return ETHOS_ERR_INVALID_ARG;
  if (bn_training && !save_bn) return ETHOS_ERR_INVALID_ARG;
  if ((htab == nullptr) != (gtab == nullptr)) return ETHOS_ERR_INVALID_ARG;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev)) != ETHOS_OK) return st;
  const ethos_dims& d = *dims;
  Carve c{static_cast<char*>(workspace), 0, workspace_bytes};
  Bwd32Scratch s;
  carve_backward_f32(c, d, htab != nullptr, &s);
  if (c.off > workspace_bytes) return ETHOS_ERR_WORKSPACE;
  cudaStream_t sm = static_cast<cudaStream_t>(stream);
  const int T = static_cast<int>(d.tokens), D = static_cast<int>(d.d_model), N = static_cast<int>(d.num_experts);
  const int H = static_cast<int>(d.num_heads), R = static_cast<int>(d.num_heads * d.top_k);
  const int dq = static_cast<int>(d.d_query), HQ = H * dq, K = static_cast<int>(d.num_sub_keys), half = dq / 2;
  const int dh = static_cast<int>(d.d_hidden), dl = static_cast<int>(d.d_latent);
  const int LDU = HQ + dh;
  const int64_t HT = static_cast<int64_t>(H) * T;
  const float invH = 1.0f / static_cast<float>(H);
  const int cb = 256;
  const int eblocks = dev->sm_count * 8;

  // accumulated outputs and the dense score gradient start at zero
  if (cudaMemsetAsync(d_w1, 0, sizeof(float) * dh * dl, sm) != cudaSuccess) return ETHOS_ERR_CUDA;
  if (cudaMemsetAsync(d_w2, 0, sizeof(float) * 2 * D * dh, sm) != cudaSuccess) return ETHOS_ERR_CUDA;
  if (cudaMemsetAsync(d_keys, 0, sizeof(float) * 2 * K * half, sm) != cudaSuccess) return ETHOS_ERR_CUDA;
  if (cudaMemsetAsync(s.cnt, 0, sizeof(int) * N, sm) != cudaSuccess) return ETHOS_ERR_CUDA;
  if (cudaMemsetAsync(s.dS, 0, sizeof(float) * 2 * HT * K, sm) != cudaSuccess) return ETHOS_ERR_CUDA;

  // (1) dhacc = dy W_v / H (W_v = net.2.weight[d:] read as [K = d][N = dh])
  if ((st = split2(dy, T, D, D, s.dy_s, sm, *dev)) != ETHOS_OK) return st;
  if ((st = split2(wv, D, dh, dh, s.wv_s, sm, *dev)) != ETHOS_OK) return st;
  const SplitOperand dyK{s.dy_s, s.dy_s + static_cast<int64_t>(T) * D, D, false};
  const SplitOperand dyM{s.dy_s, s.dy_s + static_cast<int64_t>(T) * D, D, true};
  if ((st = gemm_split(dyK, SplitOperand{s.wv_s, s.wv_s + static_cast<int64_t>(D) * dh, dh, true}, T, dh, D, s.dhacc,
                       dh, invH, false, dev_err, sm, *dev)) != ETHOS_OK)
    return st;
  // (2) dW_v = dy^T hacc / H -> d_w2[d:]
  if ((st = split2(save_hacc, T, dh, dh, s.hacc_s, sm, *dev)) != ETHOS_OK) return st;
  if ((st = gemm_split(dyM, SplitOperand{s.hacc_s, s.hacc_s + static_cast<int64_t>(T) * dh, dh, true}, D, dh, T,
                       d_w2 + static_cast<int64_t>(D) * dh, dh, invH, true, dev_err, sm, *dev)) != ETHOS_OK)
    return st;
  // (3) expert tables H and G = gelu'(E W1^T), unless the forward kept them
  if ((st = split2(latents, N, dl, dl, s.e_s, sm, *dev)) != ETHOS_OK) return st;
  if ((st = split2(w1, dh, dl, dl, s.w1_s, sm, *dev)) != ETHOS_OK) return st;
  const float* tab = htab;
  const float* gt = gtab;
  if (htab == nullptr) {
    if ((st = build_table_f32(d, latents, w1, s.e_s, s.w1_s, s.tab, s.gtab, dev_err, sm, *dev)) != ETHOS_OK)
      return st;
    tab = s.tab;
    gt = s.gtab;
  }
  // (4) per token: dw, a, ddot per selection; dxp into du[:, HQ:]
  count_launch();
  k_bwd_token_f32<<<warp_blocks(T, *dev), 256, 0, sm>>>(tab, ids, weights, save_dot, s.dhacc, s.dw, s.ca, s.cd, s.du,
                                                         LDU, HQ, T, R, N, dev_err);
  if ((st = launch_status()) != ETHOS_OK) return st;
  // (5) selections grouped by expert (counting sort)
  {
    const int64_t nsel = static_cast<int64_t>(T) * R;
    const int nblk = (N + 1023) / 1024;
    if (nblk > 1024) return ETHOS_ERR_UNSUPPORTED_SHAPE;
    count_launch();
    k_count_experts<<<eblocks, cb, 0, sm>>>(ids, nsel, N, s.cnt, dev_err);
    count_launch();
    k_scan_blocks<<<nblk, 1024, 0, sm>>>(s.cnt, N, s.offs, s.bsums);
    count_launch();
    k_scan_sums<<<1, 1024, 0, sm>>>(s.bsums, nblk, s.total);
    count_launch();
    k_scan_add<<<nblk, 1024, 0, sm>>>(s.offs, N, s.bsums, s.cursor);
    count_launch();
    k_scatter_experts<<<eblocks, cb, 0, sm>>>(ids, nsel, N, s.cursor, s.perm);
    if ((st = launch_status()) != ETHOS_OK) return st;
  }
  // (6) dP[e] = G[e] * sum over e's selections of (a dhacc_t + ddot xp_t)
  count_launch();
  k_expert_dP_f32<<<warp_blocks(N, *dev), 256, 0, sm>>>(s.offs, s.perm, s.total, s.ca, s.cd, s.dhacc, save_xp, gt,
                                                         s.dP, N, R);
  if ((st = launch_status()) != ETHOS_OK) return st;
  if ((st = split2(s.dP, N, dh, dh, s.dP_s, sm, *dev)) != ETHOS_OK) return st;
  // (7) dE = dP W1 (W1 [dh][dl] read as [K = dh][N = dl])
  const int64_t ndh = static_cast<int64_t>(N) * dh;
  if ((st = gemm_split(SplitOperand{s.dP_s, s.dP_s + ndh, dh, false},
                       SplitOperand{s.w1_s, s.w1_s + static_cast<int64_t>(dh) * dl, dl, true}, N, dl, dh, d_latents,
                       dl, 1.0f, false, dev_err, sm, *dev)) != ETHOS_OK)
    return st;
  // (8) dW1 = dP^T E (split-K over the experts)
  if ((st = gemm_split(SplitOperand{s.dP_s, s.dP_s + ndh, dh, true},
                       SplitOperand{s.e_s, s.e_s + static_cast<int64_t>(N) * dl, dl, true}, dh, dl, N, d_w1, dl, 1.0f,
                       true, dev_err, sm, *dev)) != ETHOS_OK)
    return st;
  mark(stage_events, ETHOS_BWD_STAGE_EXPERTS, sm);  // d_latents, d_w1 final
  // (9) router: softmax backward, dq^ and the dense score gradient dS
  switch (d.top_k) {
    case 4: st = launch_router_bwd_f32<4>(d, ids, weights, s.dw, keys, s.dqhat, s.dS, sm, *dev); break;
    case 8: st = launch_router_bwd_f32<8>(d, ids, weights, s.dw, keys, s.dqhat, s.dS, sm, *dev); break;
    default: st = launch_router_bwd_f32<16>(d, ids, weights, s.dw, keys, s.dqhat, s.dS, sm, *dev); break;
  }
  if (st != ETHOS_OK) return st;
  // (10) dK_p = dS_p^T q^_p over all (head, token) rows
  if ((st = split2(s.dS, 2 * HT, K, K, s.dS_s, sm, *dev)) != ETHOS_OK) return st;
  if ((st = split2(save_qhat, 2 * HT, half, half, s.qhat_s, sm, *dev)) != ETHOS_OK) return st;
  for (int p = 0; p < 2; ++p) {
    const SplitOperand a{s.dS_s + p * HT * K, s.dS_s + 2 * HT * K + p * HT * K, K, true};
    const SplitOperand b{s.qhat_s + p * HT * half, s.qhat_s + 2 * HT * half + p * HT * half, half, true};
    if ((st = gemm_split(a, b, K, half, static_cast<int>(HT), d_keys + static_cast<int64_t>(p) * K * half, half,
                         1.0f, true, dev_err, sm, *dev)) != ETHOS_OK)
      return st;
  }
  // (11) BatchNorm backward -> dq into du[:, :HQ], dbias, dgamma, dbeta
  {
    const float* mean = save_bn;
    const float* invstd = save_bn ? save_bn + HQ : nullptr;
    if (!bn_training) {
      count_launch();
      k_bn_eval_stats<<<(HQ + cb - 1) / cb, cb, 0, sm>>>(bn, HQ, bn_eps, s.stats, s.stats + HQ);
      mean = s.stats;
      invstd = s.stats + HQ;
    }
    dim3 grid_p((HQ + cb - 1) / cb, s.slabs);
    count_launch();
    k_bn_bwd_partial<<<grid_p, cb, 0, sm>>>(s.dqhat, save_qpre, mean, invstd, T, HQ, s.part);
    count_launch();
    k_bn_bwd_finalize<<<(HQ + cb - 1) / cb, cb, 0, sm>>>(s.part, s.slabs, HQ, T, bn_training, bn + HQ, mean, invstd,
                                                        d_bn + HQ, d_bn + 2 * HQ, d_bn, s.coef);
    count_launch();
    k_bn_bwd_apply_f32<<<rows_grid(HQ, T, cb, *dev), cb, 0, sm>>>(s.dqhat, save_qpre,
                                                                  reinterpret_cast<const float4*>(s.coef), T, HQ,
                                                                  s.du, LDU);
    if ((st = launch_status()) != ETHOS_OK) return st;
  }
  if ((st = split2(s.du, T, LDU, LDU, s.du_s, sm, *dev)) != ETHOS_OK) return st;
  if ((st = split2(w_cat, LDU, D, D, s.wcat_s, sm, *dev)) != ETHOS_OK) return st;
  if ((st = split2(x, T, D, D, s.x_s, sm, *dev)) != ETHOS_OK) return st;
  const int64_t tlu = static_cast<int64_t>(T) * LDU, td = static_cast<int64_t>(T) * D;
  // (12) dx = du W_cat (W_cat [ncat][d] read as [K = ncat][N = d])
  if ((st = gemm_split(SplitOperand{s.du_s, s.du_s + tlu, LDU, false},
                       SplitOperand{s.wcat_s, s.wcat_s + static_cast<int64_t>(LDU) * D, D, true}, T, D, LDU, dx, D,
                       1.0f, false, dev_err, sm, *dev)) != ETHOS_OK)
    return st;
  // (13) dWq = dq^T x   [HQ, d]
  if ((st = gemm_split(SplitOperand{s.du_s, s.du_s + tlu, LDU, true}, SplitOperand{s.x_s, s.x_s + td, D, true}, HQ, D,
                       T, d_wq, D, 1.0f, false, dev_err, sm, *dev)) != ETHOS_OK)
    return st;
  // (14) dW_u = x^T dxp -> d_w2[:d]   [d, dh]
  if ((st = gemm_split(SplitOperand{s.x_s, s.x_s + td, D, true},
                       SplitOperand{s.du_s + HQ, s.du_s + tlu + HQ, LDU, true}, D, dh, T, d_w2, dh, 1.0f, true,
                       dev_err, sm, *dev)) != ETHOS_OK)
    return st;
  mark(stage_events, ETHOS_BWD_STAGE_END, sm);
  return ETHOS_OK;
}

}  // extern "C"
