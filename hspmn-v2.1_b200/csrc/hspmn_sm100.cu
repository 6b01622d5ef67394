// C ABI of libhspmn_sm100.so (declared in include/hspmn_sm100.h): argument
// validation, launch configuration and TMA descriptor encoding for the
// router gate and selection, row gather/scatter and SQDK attention (forward and
// backward) kernels. One translation unit so all kernels share the device
// error word.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "gate.cuh"
#include "router.cuh"
#include "rows.cuh"
#include "sqdk.cuh"
#include "sqdk_bwd.cuh"

namespace hspmn {
namespace {

constexpr int kVersion = 100;  // 0.1.0
constexpr int kMaxDevices = 64;

int g_arch_ok[kMaxDevices];  // 0 unknown, 1 sm_100, -1 other

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HSPMN_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return HSPMN_ERR_DEVICE;
  int state = __atomic_load_n(&g_arch_ok[dev], __ATOMIC_ACQUIRE);
  if (state == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return HSPMN_ERR_CUDA;
    state = (major == 10 && minor == 0) ? 1 : -1;
    __atomic_store_n(&g_arch_ok[dev], state, __ATOMIC_RELEASE);
  }
  return state == 1 ? HSPMN_OK : HSPMN_ERR_DEVICE;
}

int g_sm_count[kMaxDevices];

// Streaming multiprocessors of the current device (cached per device).
int sm_count(int* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return HSPMN_ERR_CUDA;
  int n = __atomic_load_n(&g_sm_count[dev], __ATOMIC_ACQUIRE);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      return HSPMN_ERR_CUDA;
    __atomic_store_n(&g_sm_count[dev], n, __ATOMIC_RELEASE);
  }
  *out = n;
  return HSPMN_OK;
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HSPMN_OK : HSPMN_ERR_CUDA;
}

bool valid_dtype(int d) { return d == HSPMN_F32 || d == HSPMN_F16 || d == HSPMN_BF16; }
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---------------------------------------------------------------------------
// TMA descriptor encoding through the driver entry point (no libcuda link)
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 4-D tiled map over a [d3][d2][d1][d0] tensor (d0 innermost, stride 1),
// 128-byte swizzle, zero fill out of bounds. Strides in bytes.
int encode_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t dims[4],
              const uint64_t strides_bytes[3], const uint32_t box[4],
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return HSPMN_ERR_CUDA;
  cuuint64_t gd[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t gs[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, dt, 4, const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? HSPMN_OK : HSPMN_ERR_INVALID;
}

template <int HD, bool kBF16>
int launch_sqdk(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
                const SqdkParams& prm, cudaStream_t stream) {
  using L = SqdkLayout<HD>;
  auto kern = sqdk_fwd_kernel<HD, kBF16>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc) != cudaSuccess)
    return HSPMN_ERR_CUDA;
  const int64_t tiles = static_cast<int64_t>(prm.T) * prm.B * prm.Hkv;
  const int64_t grid = tiles * prm.nsplit;
  if (grid > 0x7FFFFFFF) return HSPMN_ERR_INVALID;
  kern<<<static_cast<unsigned>(grid), kSqdkThreads, L::kAlloc, stream>>>(mq, mk, mv, mo, prm);
  if (prm.nsplit > 1) {
    if (int rc = launch_status()) return rc;
    const int64_t warps = tiles * kSqdkBM;
    sqdk_combine_kernel<HD, kBF16><<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(prm);
  }
  return launch_status();
}

// Split of each tile's key blocks over several CTAs when a launch has fewer
// tiles than two per SM: enough CTAs to fill the GPU, at least ~4 blocks of
// 64 keys per split on average, at most 16 splits.
struct SqdkPlan {
  int G, QT, nsplit;
  int64_t T, tiles, ws_bytes, part_o_bytes;
};

int sqdk_plan(int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv, int64_t hd, SqdkPlan* out) {
  SqdkPlan pl;
  pl.G = static_cast<int>(H / Hkv);
  pl.QT = kSqdkBM / pl.G;
  pl.T = (K + pl.QT - 1) / pl.QT;
  pl.tiles = pl.T * B * Hkv;
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const int64_t target = 2LL * sms;
  int64_t ns = 1;
  if (pl.tiles < target) {
    ns = (target + pl.tiles - 1) / pl.tiles;
    const int64_t blocks = (S + kSqdkBN - 1) / kSqdkBN;
    ns = std::min<int64_t>(ns, std::max<int64_t>(1, blocks / 4));
    ns = std::min<int64_t>(ns, 16);
  }
  pl.nsplit = static_cast<int>(ns);
  const int64_t hdp = hd > 64 ? 128 : 64;
  pl.part_o_bytes = ns > 1 ? pl.tiles * ns * kSqdkBM * hdp * 4 : 0;
  pl.ws_bytes = ns > 1 ? pl.part_o_bytes + pl.tiles * ns * kSqdkBM * 2 * 4 : 0;
  *out = pl;
  return HSPMN_OK;
}

template <typename V>
void launch_gather(const void* src, int64_t ssb, int64_t sss, const int64_t* idx, int64_t isb, void* dst, int64_t dsb,
                   int64_t dsk, int64_t B, int64_t S, int64_t K, int64_t row_bytes, cudaStream_t stream) {
  const int64_t nrows = B * K;
  int64_t blocks = (nrows + kRowWarps - 1) / kRowWarps;
  if (blocks > 148 * 64) blocks = 148 * 64;
  gather_rows_kernel<V><<<static_cast<unsigned>(blocks), kRowThreads, 0, stream>>>(
      static_cast<const char*>(src), ssb, sss, idx, isb, static_cast<char*>(dst), dsb, dsk, B, S, K,
      row_bytes / static_cast<int64_t>(sizeof(V)));
}

template <typename V>
void launch_scatter(const void* src, int64_t ssb, int64_t ssk, const int64_t* idx, int64_t isb, void* dst,
                    int64_t dsb, int64_t dss, int64_t B, int64_t S, int64_t K, int64_t row_bytes,
                    cudaStream_t stream) {
  dim3 grid(static_cast<unsigned>((S + kScatterRowsPerCta - 1) / kScatterRowsPerCta), static_cast<unsigned>(B));
  scatter_rows_kernel<V><<<grid, kRowThreads, 0, stream>>>(static_cast<const char*>(src), ssb, ssk, idx, isb,
                                                           static_cast<char*>(dst), dsb, dss, S, K,
                                                           row_bytes / static_cast<int64_t>(sizeof(V)));
}

// widest vector (16/8/4/2 bytes) every address and stride is a multiple of
int row_vector_bytes(const void* a, const void* b, int64_t s0, int64_t s1, int64_t s2, int64_t s3,
                     int64_t row_bytes) {
  uintptr_t all = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | static_cast<uintptr_t>(s0) |
                  static_cast<uintptr_t>(s1) | static_cast<uintptr_t>(s2) | static_cast<uintptr_t>(s3) |
                  static_cast<uintptr_t>(row_bytes);
  for (int w = 16; w >= 2; w >>= 1)
    if ((all % w) == 0) return w;
  return 0;
}

}  // namespace

// Scratch of hspmn_sqdk_fwd_noalloc: the split-KV partials (unnormalised
// fp32 O, running max and row sum of each share of a tile's keys) that
// hspmn_sqdk_fwd keeps in a caller workspace. Part of the module image, so it
// exists on every device the library's kernels are loaded on; nothing in it
// needs an initial value, because each call writes every partial it reads.
static __device__ __align__(256) unsigned char g_sqdk_scratch[HSPMN_SQDK_NOALLOC_SCRATCH_BYTES];

namespace {

void* g_sqdk_scratch_addr[kMaxDevices];

// Device address of g_sqdk_scratch on the current device, looked up on the
// first call for that device and cached.
int sqdk_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return HSPMN_ERR_CUDA;
  void* p = __atomic_load_n(&g_sqdk_scratch_addr[dev], __ATOMIC_ACQUIRE);
  if (!p) {
    if (cudaGetSymbolAddress(&p, g_sqdk_scratch) != cudaSuccess || !p) return HSPMN_ERR_CUDA;
    __atomic_store_n(&g_sqdk_scratch_addr[dev], p, __ATOMIC_RELEASE);
  }
  *out = p;
  return HSPMN_OK;
}

}  // namespace
}  // namespace hspmn

using namespace hspmn;

extern "C" {

int hspmn_version(void) { return kVersion; }

const char* hspmn_strerror(int status) {
  switch (status) {
    case HSPMN_OK: return "ok";
    case HSPMN_ERR_INVALID: return "invalid argument (null pointer, size or shape)";
    case HSPMN_ERR_DTYPE: return "unsupported element type";
    case HSPMN_ERR_ALIGN: return "pointer or stride alignment not supported";
    case HSPMN_ERR_UNSUPPORTED: return "head_dim, head grouping or gate row length not supported";
    case HSPMN_ERR_CUDA: return "CUDA runtime error or launch failure";
    case HSPMN_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case HSPMN_ERR_SCRATCH: return "shape needs more split-KV scratch than the no-alloc entry's static buffer holds";
    default: return "unknown status";
  }
}

int hspmn_router_topk(const void* logits, int logits_dtype, int64_t logits_rs, const void* temp, int temp_dtype,
                      int noisy_dtype, int64_t B, int64_t S, int64_t K, int64_t* indices, int64_t indices_rs,
                      uint8_t* mask, int64_t mask_rs, void* stream) {
  if (!logits || !indices || B < 0 || S <= 0 || K < 1 || K > S || S > 0x7FFFFFFF || B > 0x7FFFFFFF)
    return HSPMN_ERR_INVALID;
  if (!valid_dtype(logits_dtype) || !valid_dtype(noisy_dtype) || (temp && !valid_dtype(temp_dtype)))
    return HSPMN_ERR_DTYPE;
  if (logits_rs < S || indices_rs < K || (mask && mask_rs < S)) return HSPMN_ERR_INVALID;
  if (B == 0) return HSPMN_OK;
  if (int rc = check_device()) return rc;
  // long rows, few of them: one cluster of kRouterClusterCtas CTAs per row
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const int nct = (S >= kRouterClusterMinS && B * kRouterClusterCtas <= sms) ? kRouterClusterCtas : 1;
  const int64_t slice = ((S + nct - 1) / nct + 7) / 8 * 8;
  const int64_t key_bytes = slice * (noisy_dtype == HSPMN_F32 ? 4 : 2);
  const bool keys_in_smem = key_bytes <= kRouterSmemKeyBytes;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto kern = keys_in_smem ? router_topk_kernel<true> : router_topk_kernel<false>;
  const size_t smem = keys_in_smem ? static_cast<size_t>(key_bytes) : 0;
  if (keys_in_smem &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kRouterSmemKeyBytes) != cudaSuccess)
    return HSPMN_ERR_CUDA;
  const int Si = static_cast<int>(S), Ki = static_cast<int>(K), slice_i = static_cast<int>(slice);
  if (nct == 1) {
    kern<<<static_cast<unsigned>(B), kRouterThreads, smem, st>>>(logits, logits_dtype, logits_rs, temp, temp_dtype,
                                                                 noisy_dtype, Si, Ki, indices, indices_rs, mask,
                                                                 mask_rs, slice_i);
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(B * nct));
    cfg.blockDim = dim3(kRouterThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(nct);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, logits, logits_dtype, logits_rs, temp, temp_dtype, noisy_dtype, Si, Ki,
                           indices, indices_rs, mask, mask_rs, slice_i) != cudaSuccess)
      return HSPMN_ERR_CUDA;
  }
  return launch_status();
}

int hspmn_gate_logits(const void* x, int x_dtype, int64_t x_sb, int64_t x_ss, const void* weight,
                      const void* bias, int64_t B, int64_t S, int64_t D, float* logits, int64_t logits_rs,
                      void* stream) {
  if (!x || !weight || !logits || B < 0 || S < 1 || D < 1 || x_sb < 0 || x_ss < 0 || logits_rs < S)
    return HSPMN_ERR_INVALID;
  if (!valid_dtype(x_dtype)) return HSPMN_ERR_DTYPE;
  const int64_t es = x_dtype == HSPMN_F32 ? 4 : 2;
  const int64_t per_vec = 16 / es;
  if (D % per_vec != 0 || D / per_vec > 0x7FFFFFFF) return HSPMN_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(weight)) % 16 != 0 ||
      (x_sb * es) % 16 != 0 || (x_ss * es) % 16 != 0)
    return HSPMN_ERR_ALIGN;
  if (B == 0) return HSPMN_OK;
  if (int rc = check_device()) return rc;
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  auto kern = x_dtype == HSPMN_F32   ? gate_logits_kernel<float>
              : x_dtype == HSPMN_F16 ? gate_logits_kernel<__half>
                                     : gate_logits_kernel<__nv_bfloat16>;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGateThreads, 0) != cudaSuccess || per_sm < 1)
    return HSPMN_ERR_CUDA;
  const int64_t need = (B * S + kGateWarps - 1) / kGateWarps;
  const int64_t grid = std::min<int64_t>(need, static_cast<int64_t>(sms) * per_sm);
  kern<<<static_cast<unsigned>(grid), kGateThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(x), x_sb * es, x_ss * es, static_cast<const uint4*>(weight), bias, B, S,
      static_cast<int>(D / per_vec), logits, logits_rs);
  return launch_status();
}

int hspmn_gather_rows(const void* src, int64_t src_sb, int64_t src_ss, const int64_t* idx, int64_t idx_sb,
                      void* dst, int64_t dst_sb, int64_t dst_sk, int64_t B, int64_t S, int64_t K, int64_t row_bytes,
                      void* stream) {
  if (!src || !idx || !dst || B < 0 || S < 1 || K < 0 || row_bytes <= 0) return HSPMN_ERR_INVALID;
  if (src_sb < 0 || src_ss < 0 || dst_sb < 0 || dst_sk < 0 || idx_sb < K) return HSPMN_ERR_INVALID;
  if (B == 0 || K == 0) return HSPMN_OK;
  const int vec = row_vector_bytes(src, dst, src_sb, src_ss, dst_sb, dst_sk, row_bytes);
  if (vec == 0) return HSPMN_ERR_ALIGN;
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (vec) {
    case 16: launch_gather<uint4>(src, src_sb, src_ss, idx, idx_sb, dst, dst_sb, dst_sk, B, S, K, row_bytes, st); break;
    case 8: launch_gather<uint2>(src, src_sb, src_ss, idx, idx_sb, dst, dst_sb, dst_sk, B, S, K, row_bytes, st); break;
    case 4: launch_gather<unsigned>(src, src_sb, src_ss, idx, idx_sb, dst, dst_sb, dst_sk, B, S, K, row_bytes, st); break;
    case 2: launch_gather<unsigned short>(src, src_sb, src_ss, idx, idx_sb, dst, dst_sb, dst_sk, B, S, K, row_bytes, st); break;
    default: return HSPMN_ERR_ALIGN;
  }
  return launch_status();
}

int hspmn_scatter_rows(const void* src, int64_t src_sb, int64_t src_sk, const int64_t* idx, int64_t idx_sb,
                       void* dst, int64_t dst_sb, int64_t dst_ss, int64_t B, int64_t S, int64_t K, int64_t row_bytes,
                       void* stream) {
  if (!dst || B < 0 || S < 1 || K < 0 || row_bytes <= 0 || K > S) return HSPMN_ERR_INVALID;
  if ((K > 0 && (!src || !idx || idx_sb < K)) || src_sb < 0 || src_sk < 0 || dst_sb < 0 || dst_ss < 0)
    return HSPMN_ERR_INVALID;
  if (B == 0) return HSPMN_OK;
  if (B > 65535) return HSPMN_ERR_INVALID;
  const int vec = row_vector_bytes(src ? src : dst, dst, src_sb, src_sk, dst_sb, dst_ss, row_bytes);
  if (vec == 0) return HSPMN_ERR_ALIGN;
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (vec) {
    case 16: launch_scatter<uint4>(src, src_sb, src_sk, idx, idx_sb, dst, dst_sb, dst_ss, B, S, K, row_bytes, st); break;
    case 8: launch_scatter<uint2>(src, src_sb, src_sk, idx, idx_sb, dst, dst_sb, dst_ss, B, S, K, row_bytes, st); break;
    case 4: launch_scatter<unsigned>(src, src_sb, src_sk, idx, idx_sb, dst, dst_sb, dst_ss, B, S, K, row_bytes, st); break;
    case 2: launch_scatter<unsigned short>(src, src_sb, src_sk, idx, idx_sb, dst, dst_sb, dst_ss, B, S, K, row_bytes, st); break;
    default: return HSPMN_ERR_ALIGN;
  }
  return launch_status();
}

int hspmn_rope_gather_rows(const void* src, int64_t src_sb, int64_t src_ss, int src_by_position, const int64_t* idx,
                           int64_t idx_sb, const void* cos_tab, const void* sin_tab, int64_t tab_ss, void* dst,
                           int64_t dst_sb, int64_t dst_sk, int64_t B, int64_t S, int64_t K, int64_t H, int64_t hd,
                           int dtype, void* stream) {
  if (!src || !idx || !cos_tab || !sin_tab || !dst || B < 0 || S < 1 || K < 0 || H < 1 || hd < 2)
    return HSPMN_ERR_INVALID;
  if (!valid_dtype(dtype)) return HSPMN_ERR_DTYPE;
  // idx_sb may be 0: every sequence reads the same positions (e.g. all of them)
  if (idx_sb < 0 || src_sb < 0 || src_ss < 0 || dst_sb < 0 || dst_sk < 0 || tab_ss < hd) return HSPMN_ERR_INVALID;
  if (B == 0 || K == 0) return HSPMN_OK;
  if (B * K > 0x7FFFFFFFLL * kRowWarps || H * hd > 0x7FFFFFFF) return HSPMN_ERR_INVALID;
  const int64_t es = dtype == HSPMN_F32 ? 4 : 2;
  const int64_t vec = 16 / es;
  if (hd % (2 * vec) != 0) return HSPMN_ERR_UNSUPPORTED;
  if (!aligned(src, 16) || !aligned(dst, 16) || !aligned(cos_tab, 16) || !aligned(sin_tab, 16) ||
      (src_sb * es) % 16 || (src_ss * es) % 16 || (dst_sb * es) % 16 || (dst_sk * es) % 16 || (tab_ss * es) % 16)
    return HSPMN_ERR_ALIGN;
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t blocks = (B * K + kRowWarps - 1) / kRowWarps;
  if (blocks > 148 * 64) blocks = 148 * 64;
  const unsigned g = static_cast<unsigned>(blocks);
#define HSPMN_ROPE_LAUNCH(T)                                                                                       \
  rope_gather_rows_kernel<T><<<g, kRowThreads, 0, st>>>(                                                          \
      static_cast<const T*>(src), src_sb, src_ss, src_by_position, idx, idx_sb, static_cast<const T*>(cos_tab),     \
      static_cast<const T*>(sin_tab), tab_ss, static_cast<T*>(dst), dst_sb, dst_sk, B, S, K, static_cast<int>(H),   \
      static_cast<int>(hd))
  if (dtype == HSPMN_BF16) HSPMN_ROPE_LAUNCH(__nv_bfloat16);
  else if (dtype == HSPMN_F16) HSPMN_ROPE_LAUNCH(__half);
  else HSPMN_ROPE_LAUNCH(float);
#undef HSPMN_ROPE_LAUNCH
  return launch_status();
}

int hspmn_rope_rows(const void* src, int64_t src_sb, int64_t src_ss, const void* cos_tab, const void* sin_tab,
                    int64_t tab_ss, int64_t tab_rows, int64_t pos0, void* dst, int64_t dst_sb, int64_t dst_ss,
                    int64_t B, int64_t S, int64_t H, int64_t hd, int dtype, void* stream) {
  if (!src || !cos_tab || !sin_tab || !dst || B < 0 || S < 0 || H < 1 || hd < 2 || pos0 < 0)
    return HSPMN_ERR_INVALID;
  if (!valid_dtype(dtype)) return HSPMN_ERR_DTYPE;
  if (src_sb < 0 || src_ss < 0 || dst_sb < 0 || dst_ss < 0 || tab_ss < hd || pos0 + S > tab_rows)
    return HSPMN_ERR_INVALID;
  if (B == 0 || S == 0) return HSPMN_OK;
  if (H * hd > 0x7FFFFFFF) return HSPMN_ERR_INVALID;
  const int64_t es = dtype == HSPMN_F32 ? 4 : 2;
  const int64_t vec = 16 / es;
  if (hd % (2 * vec) != 0) return HSPMN_ERR_UNSUPPORTED;
  if (!aligned(src, 16) || !aligned(dst, 16) || !aligned(cos_tab, 16) || !aligned(sin_tab, 16) ||
      (src_sb * es) % 16 || (src_ss * es) % 16 || (dst_sb * es) % 16 || (dst_ss * es) % 16 || (tab_ss * es) % 16)
    return HSPMN_ERR_ALIGN;
  if (int rc = check_device()) return rc;
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t warps = (B * S + 1) / 2;
  int64_t blocks = (warps + kRowWarps - 1) / kRowWarps;
  blocks = std::min<int64_t>(blocks, static_cast<int64_t>(sms) * 8);
  const unsigned g = static_cast<unsigned>(blocks);
#define HSPMN_ROPE_ROWS_LAUNCH(T)                                                                                    \
  rope_rows_kernel<T><<<g, kRowThreads, 0, st>>>(static_cast<const T*>(src), src_sb, src_ss,                        \
                                                 static_cast<const T*>(cos_tab), static_cast<const T*>(sin_tab),     \
                                                 tab_ss, pos0, static_cast<T*>(dst), dst_sb, dst_ss, B, S,           \
                                                 static_cast<int>(H), static_cast<int>(hd))
  if (dtype == HSPMN_BF16) HSPMN_ROPE_ROWS_LAUNCH(__nv_bfloat16);
  else if (dtype == HSPMN_F16) HSPMN_ROPE_ROWS_LAUNCH(__half);
  else HSPMN_ROPE_ROWS_LAUNCH(float);
#undef HSPMN_ROPE_ROWS_LAUNCH
  return launch_status();
}

int hspmn_scatter_add_rows(const void* src, int64_t src_sb, int64_t src_sk, const int64_t* idx, int64_t idx_sb,
                           void* dst, int64_t dst_sb, int64_t dst_ss, int64_t B, int64_t S, int64_t K,
                           int64_t row_elems, int dtype, void* stream) {
  if (!src || !idx || !dst || B < 0 || S < 1 || K < 0 || row_elems < 1) return HSPMN_ERR_INVALID;
  if (!valid_dtype(dtype)) return HSPMN_ERR_DTYPE;
  if (idx_sb < K || src_sb < 0 || src_sk < 0 || dst_sb < 0 || dst_ss < 0) return HSPMN_ERR_INVALID;
  if (B == 0 || K == 0) return HSPMN_OK;
  const int64_t es = dtype == HSPMN_F32 ? 4 : 2;
  if ((row_elems * es) % 16 || !aligned(src, 16) || !aligned(dst, 16) || (src_sb * es) % 16 || (src_sk * es) % 16 ||
      (dst_sb * es) % 16 || (dst_ss * es) % 16)
    return HSPMN_ERR_ALIGN;
  if (int rc = check_device()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t blocks = (B * K + kRowWarps - 1) / kRowWarps;
  if (blocks > 148 * 64) blocks = 148 * 64;
  const unsigned g = static_cast<unsigned>(blocks);
#define HSPMN_SCATTER_ADD_LAUNCH(T)                                                                              \
  scatter_add_rows_kernel<T><<<g, kRowThreads, 0, st>>>(static_cast<const T*>(src), src_sb, src_sk, idx, idx_sb, \
                                                        static_cast<T*>(dst), dst_sb, dst_ss, B, S, K, row_elems)
  if (dtype == HSPMN_BF16) HSPMN_SCATTER_ADD_LAUNCH(__nv_bfloat16);
  else if (dtype == HSPMN_F16) HSPMN_SCATTER_ADD_LAUNCH(__half);
  else HSPMN_SCATTER_ADD_LAUNCH(float);
#undef HSPMN_SCATTER_ADD_LAUNCH
  return launch_status();
}

}  // extern "C"

namespace {

int sqdk_fwd_impl(const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
                  const int64_t* vs, const int64_t* idx, int64_t idx_sb, int64_t idx_sk, void* o, const int64_t* os,
                  float* lse, int64_t lse_sb, int64_t lse_sk, int64_t B, int64_t K, int64_t S, int64_t H,
                  int64_t Hkv, int64_t hd, int dtype, float sm_scale, void* workspace, size_t workspace_bytes,
                  bool static_scratch, void* stream) {
  if (!q || !k || !v || !idx || !o || !qs || !ks || !vs || !os) return HSPMN_ERR_INVALID;
  if (lse && (lse_sk < H || lse_sb < 0)) return HSPMN_ERR_INVALID;
  if (B < 0 || K < 0 || S < 1 || H < 1 || Hkv < 1 || !(sm_scale > 0.0f) || !std::isfinite(sm_scale))
    return HSPMN_ERR_INVALID;
  if (dtype != HSPMN_BF16 && dtype != HSPMN_F16) return HSPMN_ERR_DTYPE;
  if (hd < 8 || hd > 128 || hd % 8 != 0) return HSPMN_ERR_UNSUPPORTED;
  if (H % Hkv != 0 || H / Hkv > kSqdkBM) return HSPMN_ERR_UNSUPPORTED;
  if (B == 0 || K == 0) return HSPMN_OK;
  if (B > 0x7FFFFFFF || K > 0x7FFFFFFF || S > 0x7FFFFFFF) return HSPMN_ERR_INVALID;
  const int64_t es = 2;
  if (qs[3] != 1 || ks[3] != 1 || vs[3] != 1 || os[3] != 1) return HSPMN_ERR_ALIGN;
  for (int i = 0; i < 3; ++i) {
    if ((qs[i] * es) % 16 || (ks[i] * es) % 16 || (vs[i] * es) % 16 || (os[i] * es) % 16) return HSPMN_ERR_ALIGN;
    if (qs[i] <= 0 || ks[i] <= 0 || vs[i] <= 0 || os[i] <= 0) return HSPMN_ERR_INVALID;
  }
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(o, 16)) return HSPMN_ERR_ALIGN;
  if (int rc = check_device()) return rc;

  SqdkPlan pl;
  if (int rc = sqdk_plan(B, K, S, H, Hkv, hd, &pl)) return rc;
  if (static_scratch) {
    // hspmn_sqdk_fwd_noalloc: the split-KV partials go to the library's own
    // device array, looked up only for launches that split
    if (pl.ws_bytes > static_cast<int64_t>(HSPMN_SQDK_NOALLOC_SCRATCH_BYTES)) return HSPMN_ERR_SCRATCH;
    if (pl.ws_bytes > 0) {
      if (int rc = sqdk_scratch(&workspace)) return rc;
      workspace_bytes = HSPMN_SQDK_NOALLOC_SCRATCH_BYTES;
    }
  }
  if (pl.ws_bytes > 0 && (!workspace || workspace_bytes < static_cast<size_t>(pl.ws_bytes)))
    return HSPMN_ERR_INVALID;
  if (pl.ws_bytes > 0 && !aligned(workspace, 16)) return HSPMN_ERR_ALIGN;
  const int G = pl.G;
  const int QT = pl.QT;
  const int64_t T = pl.T;
  const CUtensorMapDataType dt =
      dtype == HSPMN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;

  CUtensorMap mq, mk, mv, mo;
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(H), static_cast<uint64_t>(K),
                              static_cast<uint64_t>(B)};
    const uint64_t str[3] = {static_cast<uint64_t>(qs[2] * es), static_cast<uint64_t>(qs[1] * es),
                             static_cast<uint64_t>(qs[0] * es)};
    const uint32_t box[4] = {64u, static_cast<uint32_t>(G), static_cast<uint32_t>(QT), 1u};
    if (int rc = encode_4d(&mq, q, dt, dims, str, box)) return rc;
    // the output tile has the query tile's shape; the epilogue stores it with this map
    const uint64_t ostr[3] = {static_cast<uint64_t>(os[2] * es), static_cast<uint64_t>(os[1] * es),
                              static_cast<uint64_t>(os[0] * es)};
    if (int rc = encode_4d(&mo, o, dt, dims, ostr, box)) return rc;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(Hkv), static_cast<uint64_t>(S),
                              static_cast<uint64_t>(B)};
    const uint32_t box[4] = {64u, 1u, static_cast<uint32_t>(kSqdkBN), 1u};
    const uint64_t sk[3] = {static_cast<uint64_t>(ks[2] * es), static_cast<uint64_t>(ks[1] * es),
                            static_cast<uint64_t>(ks[0] * es)};
    const uint64_t sv[3] = {static_cast<uint64_t>(vs[2] * es), static_cast<uint64_t>(vs[1] * es),
                            static_cast<uint64_t>(vs[0] * es)};
    if (int rc = encode_4d(&mk, k, dt, dims, sk, box)) return rc;
    if (int rc = encode_4d(&mv, v, dt, dims, sv, box)) return rc;
  }
  SqdkParams prm;
  prm.idx = idx;
  prm.hd = static_cast<int>(hd);
  prm.nsplit = pl.nsplit;
  prm.part_o = pl.ws_bytes > 0 ? static_cast<float*>(workspace) : nullptr;
  prm.part_ml = pl.ws_bytes > 0 ? reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.part_o_bytes) : nullptr;
  prm.idx_sb = idx_sb;
  prm.idx_sk = idx_sk;
  prm.o = o;
  prm.o_sb = os[0];
  prm.o_sk = os[1];
  prm.o_sh = os[2];
  prm.B = static_cast<int>(B);
  prm.K = static_cast<int>(K);
  prm.S = static_cast<int>(S);
  prm.H = static_cast<int>(H);
  prm.Hkv = static_cast<int>(Hkv);
  prm.G = G;
  prm.QT = QT;
  prm.T = static_cast<int>(T);
  prm.scale_log2 = sm_scale * 1.4426950408889634f;
  prm.lse = lse;
  prm.lse_sb = lse_sb;
  prm.lse_sk = lse_sk;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (hd > 64)
    return dtype == HSPMN_BF16 ? launch_sqdk<128, true>(mq, mk, mv, mo, prm, st)
                              : launch_sqdk<128, false>(mq, mk, mv, mo, prm, st);
  return dtype == HSPMN_BF16 ? launch_sqdk<64, true>(mq, mk, mv, mo, prm, st)
                             : launch_sqdk<64, false>(mq, mk, mv, mo, prm, st);
}

}  // namespace

extern "C" {

int hspmn_sqdk_fwd(const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
                   const int64_t* vs, const int64_t* idx, int64_t idx_sb, int64_t idx_sk, void* o,
                   const int64_t* os, int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv, int64_t hd,
                   int dtype, float sm_scale, void* workspace, size_t workspace_bytes, void* stream) {
  return sqdk_fwd_impl(q, qs, k, ks, v, vs, idx, idx_sb, idx_sk, o, os, nullptr, 0, 0, B, K, S, H, Hkv, hd, dtype,
                       sm_scale, workspace, workspace_bytes, false, stream);
}

int hspmn_sqdk_fwd_lse(const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
                       const int64_t* vs, const int64_t* idx, int64_t idx_sb, int64_t idx_sk, void* o,
                       const int64_t* os, float* lse, int64_t lse_sb, int64_t lse_sk, int64_t B, int64_t K,
                       int64_t S, int64_t H, int64_t Hkv, int64_t hd, int dtype, float sm_scale, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (!lse) return HSPMN_ERR_INVALID;
  return sqdk_fwd_impl(q, qs, k, ks, v, vs, idx, idx_sb, idx_sk, o, os, lse, lse_sb, lse_sk, B, K, S, H, Hkv, hd,
                       dtype, sm_scale, workspace, workspace_bytes, false, stream);
}

int64_t hspmn_sqdk_bwd_workspace_size(int64_t B, int64_t K, int64_t H, int64_t hd) {
  if (B < 1 || K < 1 || H < 1 || hd < 1) return 0;
  const int64_t delta = (B * K * H * 4 + 255) / 256 * 256;
  return delta + B * K * H * hd * 4;
}

int hspmn_sqdk_bwd(const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
                   const int64_t* vs, const int64_t* idx, int64_t idx_sb, int64_t idx_sk, const void* o,
                   const int64_t* os, const void* d_o, const int64_t* dos, const float* lse, int64_t lse_sb,
                   int64_t lse_sk, void* dq, const int64_t* dqs, void* dk, const int64_t* dks, void* dv,
                   const int64_t* dvs, int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv, int64_t hd,
                   int dtype, float sm_scale, void* workspace, size_t workspace_bytes, void* stream) {
  // with K == 0 the query-side tensors are empty (their pointers may be null)
  if (!k || !v || !dk || !dv) return HSPMN_ERR_INVALID;
  if (!qs || !ks || !vs || !os || !dos || !dqs || !dks || !dvs) return HSPMN_ERR_INVALID;
  if (B < 0 || K < 0 || S < 1 || H < 1 || Hkv < 1 || !(sm_scale > 0.0f) || !std::isfinite(sm_scale))
    return HSPMN_ERR_INVALID;
  if (K > 0 && (!q || !idx || !o || !d_o || !lse || !dq)) return HSPMN_ERR_INVALID;
  if (dtype != HSPMN_BF16 && dtype != HSPMN_F16) return HSPMN_ERR_DTYPE;
  if (hd < 8 || hd > kBwdHD || hd % 8 != 0) return HSPMN_ERR_UNSUPPORTED;
  if (H % Hkv != 0 || H / Hkv > kBwdRows) return HSPMN_ERR_UNSUPPORTED;
  if (B > 0x7FFFFFFF || K > 0x7FFFFFFF || S > 0x7FFFFFFF) return HSPMN_ERR_INVALID;
  if (K > 0 && (lse_sb != K * H || lse_sk != H)) return HSPMN_ERR_INVALID;  // lse dense [B,K,H], like Delta
  const int64_t es = 2;
  // key-side tensors always; query-side ones only when there are queries
  const int64_t* key_s[4] = {ks, vs, dks, dvs};
  const int64_t* query_s[4] = {qs, os, dos, dqs};
  for (const int64_t* st : key_s) {
    if (st[3] != 1) return HSPMN_ERR_ALIGN;
    for (int i = 0; i < 3; ++i) {
      if ((st[i] * es) % 16) return HSPMN_ERR_ALIGN;
      if (st[i] <= 0) return HSPMN_ERR_INVALID;
    }
  }
  if (K > 0) {
    for (const int64_t* st : query_s) {
      if (st[3] != 1) return HSPMN_ERR_ALIGN;
      for (int i = 0; i < 3; ++i)
        if (st[i] <= 0) return HSPMN_ERR_INVALID;
    }
    for (int i = 0; i < 3; ++i)
      if ((qs[i] * es) % 16 || (dos[i] * es) % 16) return HSPMN_ERR_ALIGN;
  }
  // (a null pointer counts as aligned)
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(d_o, 16) || !aligned(dk, 16) ||
      !aligned(dv, 16))
    return HSPMN_ERR_ALIGN;
  if (B == 0) return HSPMN_OK;
  // K == 0: no query block reaches any key block; the kernel writes zero dK / dV
  const int64_t need = K > 0 ? hspmn_sqdk_bwd_workspace_size(B, K, H, hd) : 0;
  if (need > 0 && (!workspace || workspace_bytes < static_cast<size_t>(need))) return HSPMN_ERR_INVALID;
  if (need > 0 && !aligned(workspace, 16)) return HSPMN_ERR_ALIGN;
  if (int rc = check_device()) return rc;
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = static_cast<int>(H / Hkv);
  const int QTb = kBwdRows / G;
  float* delta = static_cast<float*>(workspace);
  float* dq_acc = K > 0 ? reinterpret_cast<float*>(static_cast<char*>(workspace) + (B * K * H * 4 + 255) / 256 * 256)
                        : nullptr;
  if (K > 0) {
    if (cudaMemsetAsync(dq_acc, 0, static_cast<size_t>(B * K * H * hd * 4), st) != cudaSuccess) return HSPMN_ERR_CUDA;
    const int64_t rows = B * K * H;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((rows + 7) / 8, static_cast<int64_t>(sms) * 16));
    if (dtype == HSPMN_BF16)
      sqdk_bwd_delta_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
          static_cast<const __nv_bfloat16*>(o), os[0], os[1], os[2], static_cast<const __nv_bfloat16*>(d_o), dos[0],
          dos[1], dos[2], delta, static_cast<int>(B), static_cast<int>(K), static_cast<int>(H), static_cast<int>(hd));
    else
      sqdk_bwd_delta_kernel<__half><<<grid, 256, 0, st>>>(
          static_cast<const __half*>(o), os[0], os[1], os[2], static_cast<const __half*>(d_o), dos[0], dos[1], dos[2],
          delta, static_cast<int>(B), static_cast<int>(K), static_cast<int>(H), static_cast<int>(hd));
    if (int rc = launch_status()) return rc;
  }
  const CUtensorMapDataType dt =
      dtype == HSPMN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv, mdo, mdk, mdv;
  std::memset(&mq, 0, sizeof(mq));
  std::memset(&mdo, 0, sizeof(mdo));
  if (K > 0) {
    const uint64_t dims[4] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(H), static_cast<uint64_t>(K),
                              static_cast<uint64_t>(B)};
    const uint32_t box[4] = {64u, static_cast<uint32_t>(G), static_cast<uint32_t>(QTb), 1u};
    const uint64_t sq[3] = {static_cast<uint64_t>(qs[2] * es), static_cast<uint64_t>(qs[1] * es),
                            static_cast<uint64_t>(qs[0] * es)};
    const uint64_t sd[3] = {static_cast<uint64_t>(dos[2] * es), static_cast<uint64_t>(dos[1] * es),
                            static_cast<uint64_t>(dos[0] * es)};
    if (int rc = encode_4d(&mq, q, dt, dims, sq, box)) return rc;
    if (int rc = encode_4d(&mdo, d_o, dt, dims, sd, box)) return rc;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(Hkv), static_cast<uint64_t>(S),
                              static_cast<uint64_t>(B)};
    const uint32_t box[4] = {64u, 1u, static_cast<uint32_t>(kBwdKeys), 1u};
    const uint64_t sk[3] = {static_cast<uint64_t>(ks[2] * es), static_cast<uint64_t>(ks[1] * es),
                            static_cast<uint64_t>(ks[0] * es)};
    const uint64_t sv[3] = {static_cast<uint64_t>(vs[2] * es), static_cast<uint64_t>(vs[1] * es),
                            static_cast<uint64_t>(vs[0] * es)};
    if (int rc = encode_4d(&mk, k, dt, dims, sk, box)) return rc;
    if (int rc = encode_4d(&mv, v, dt, dims, sv, box)) return rc;
    // dV / dK leave the kernel through TMA stores of the same 64 x 128-key tile
    const uint64_t sdk[3] = {static_cast<uint64_t>(dks[2] * es), static_cast<uint64_t>(dks[1] * es),
                             static_cast<uint64_t>(dks[0] * es)};
    const uint64_t sdv[3] = {static_cast<uint64_t>(dvs[2] * es), static_cast<uint64_t>(dvs[1] * es),
                             static_cast<uint64_t>(dvs[0] * es)};
    if (int rc = encode_4d(&mdk, dk, dt, dims, sdk, box)) return rc;
    if (int rc = encode_4d(&mdv, dv, dt, dims, sdv, box)) return rc;
  }
  // the fp32 dq accumulator, added into per query block with bulk tensor reduces
  CUtensorMap mdq;
  std::memset(&mdq, 0, sizeof(mdq));
  if (K > 0) {
    const uint64_t dims[4] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(H), static_cast<uint64_t>(K),
                              static_cast<uint64_t>(B)};
    const uint64_t sq[3] = {static_cast<uint64_t>(hd * 4), static_cast<uint64_t>(H * hd * 4),
                            static_cast<uint64_t>(K * H * hd * 4)};
    const uint32_t box[4] = {64u, static_cast<uint32_t>(G), static_cast<uint32_t>(QTb), 1u};
    if (int rc = encode_4d(&mdq, dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dims, sq, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  }
  SqdkBwdParams prm;
  prm.idx = idx;
  prm.idx_sb = idx_sb;
  prm.idx_sk = idx_sk;
  prm.lse = lse;
  prm.delta = delta;
  prm.row_sb = K * H;
  prm.row_sk = H;
  prm.dq = dq_acc;
  prm.dk = dk;
  prm.dv = dv;
  prm.dk_sb = dks[0];
  prm.dk_ss = dks[1];
  prm.dk_sh = dks[2];
  prm.dv_sb = dvs[0];
  prm.dv_ss = dvs[1];
  prm.dv_sh = dvs[2];
  prm.B = static_cast<int>(B);
  prm.K = static_cast<int>(K);
  prm.S = static_cast<int>(S);
  prm.H = static_cast<int>(H);
  prm.Hkv = static_cast<int>(Hkv);
  prm.G = G;
  prm.QTb = QTb;
  prm.hd = static_cast<int>(hd);
  prm.nkb = static_cast<int>((S + kBwdKeys - 1) / kBwdKeys);
  // about one SM-count of CTAs per chunk of (sequence, head) pairs
  prm.chunk = std::max(1, std::min(static_cast<int>(B * Hkv), sms / prm.nkb));
  prm.scale = sm_scale;
  prm.scale_log2 = sm_scale * 1.4426950408889634f;
  const int64_t grid = static_cast<int64_t>(prm.nkb) * B * Hkv;
  if (grid > 0x7FFFFFFF) return HSPMN_ERR_INVALID;
  auto kern = dtype == HSPMN_BF16 ? sqdk_bwd_kernel<true> : sqdk_bwd_kernel<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SqdkBwdLayout::kAlloc) != cudaSuccess)
    return HSPMN_ERR_CUDA;
  kern<<<static_cast<unsigned>(grid), kBwdThreads, SqdkBwdLayout::kAlloc, st>>>(mq, mk, mv, mdo, mdq, mdv, mdk,
                                                                                 prm);
  if (int rc = launch_status()) return rc;
  if (K > 0) {
    const int64_t n = B * K * H * hd;
    const unsigned g2 = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(sms) * 32));
    if (dtype == HSPMN_BF16)
      sqdk_bwd_dq_cast_kernel<__nv_bfloat16><<<g2, 256, 0, st>>>(dq_acc, static_cast<__nv_bfloat16*>(dq), dqs[0],
                                                                  dqs[1], dqs[2], static_cast<int>(B),
                                                                  static_cast<int>(K), static_cast<int>(H),
                                                                  static_cast<int>(hd), sm_scale);
    else
      sqdk_bwd_dq_cast_kernel<__half><<<g2, 256, 0, st>>>(dq_acc, static_cast<__half*>(dq), dqs[0], dqs[1], dqs[2],
                                                           static_cast<int>(B), static_cast<int>(K),
                                                           static_cast<int>(H), static_cast<int>(hd), sm_scale);
  }
  return launch_status();
}

int64_t hspmn_sqdk_workspace_size(int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv, int64_t hd) {
  if (B < 1 || K < 1 || S < 1 || H < 1 || Hkv < 1 || H % Hkv != 0 || H / Hkv > kSqdkBM) return 0;
  SqdkPlan pl;
  if (sqdk_plan(B, K, S, H, Hkv, hd, &pl) != HSPMN_OK) return -1;
  return pl.ws_bytes;
}

int hspmn_sqdk_fwd_noalloc(const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
                           const int64_t* vs, const int64_t* idx, int64_t idx_sb, int64_t idx_sk, void* o,
                           const int64_t* os, int64_t B, int64_t K, int64_t S, int64_t H, int64_t Hkv, int64_t hd,
                           int dtype, float sm_scale, void* stream) {
  // the same validation, in the same order, as hspmn_sqdk_fwd; the static
  // scratch stands in for the caller's workspace
  return sqdk_fwd_impl(q, qs, k, ks, v, vs, idx, idx_sb, idx_sk, o, os, nullptr, 0, 0, B, K, S, H, Hkv, hd, dtype,
                       sm_scale, nullptr, 0, true, stream);
}

int hspmn_device_errors(unsigned* bits, int clear, void* stream) {
  if (!bits) return HSPMN_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return HSPMN_ERR_CUDA;
  if (cudaMemcpyFromSymbol(bits, g_device_errors, sizeof(unsigned)) != cudaSuccess) return HSPMN_ERR_CUDA;
  if (clear) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_device_errors, &zero, sizeof(unsigned)) != cudaSuccess) return HSPMN_ERR_CUDA;
  }
  return HSPMN_OK;
}

}  // extern "C"
