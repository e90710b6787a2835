// libh3b200: the C ABI (include/h3b200.h) over the sm_100a kernels.  One translation unit: every kernel header is
// included here, so the device status word and the kernels live in one module.  Host code validates arguments,
// builds TMA tensor maps (cuTensorMapEncodeTiled, fetched from the driver at first use) and launches on the
// caller's stream.  Nothing here allocates device memory.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "attention.cuh"
#include "elementwise.cuh"
#include "gemm_nvfp4.cuh"
#include "h3b200.h"

using namespace h3;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return H3_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ------------------------------------------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
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

// 2-D byte matrix [rows, cols] (row stride `ld` bytes) read in boxes of box_cols (<= 128) x box_rows, 128-byte swizzle.
int make_map_u8(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                uint32_t box_rows, const char* what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(H3_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable from the driver", what);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(H3_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return H3_OK;
}

// A tiled scale buffer (h3_sf_tiled_bytes layout) as rows of 2048 bytes -- the scales of 128 matrix rows for one
// 256-element K tile, contiguous -- read one row per box (256 eight-byte elements, no swizzle).
int make_map_sf_rows(CUtensorMap* map, const void* base, uint64_t rows, const char* what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(H3_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable from the driver", what);
  cuuint64_t dims[2] = {256, rows};
  cuuint64_t strides[1] = {2048};
  cuuint32_t box[2] = {256, 1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(H3_ERR_CUDA, "%s: cuTensorMapEncodeTiled (scales) failed (%d)", what, (int)r);
  return H3_OK;
}

// Opt a kernel into more than 48 KB of dynamic shared memory once per device.
template <typename K>
int smem_optin(K kernel, int bytes, unsigned* done_mask, const char* what) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 32 && (__atomic_load_n(done_mask, __ATOMIC_RELAXED) >> dev) & 1u) return H3_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", what, cudaGetErrorString(e));
  if (dev < 32) __atomic_fetch_or(done_mask, 1u << dev, __ATOMIC_RELAXED);
  return H3_OK;
}

unsigned g_optin_attn[2] = {0, 0};   // [NT - 1]
#ifndef H3_GEMM_PAIR
#define H3_GEMM_PAIR 0
#endif

// Streaming multiprocessors of the current device (cached per device).
int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

unsigned g_optin_gemm[2][5] = {};

template <int BN, int EPI>
int launch_gemm_t(int grid, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& p, cudaStream_t st) {
  int rc = smem_optin(gemm_nvfp4_kernel<BN, EPI>, GemmSmem<BN>::TOTAL, &g_optin_gemm[BN == 256][EPI], "h3_gemm_nvfp4");
  if (rc) return rc;
  gemm_nvfp4_kernel<BN, EPI><<<grid, kGemmThreads(EPI), GemmSmem<BN>::TOTAL, st>>>(ta, tb, p);
  return H3_OK;
}

unsigned g_optin_pair[5] = {};

// CTA pairs: a cluster of two CTAs per output tile (tcgen05 cta_group::2).
template <int EPI>
int launch_gemm_pair_t(int grid, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa,
                       const CUtensorMap& tsb, const GemmArgs& p, cudaStream_t st) {
  int rc = smem_optin(gemm_nvfp4_pair_kernel<EPI>, GemmPairSmem::TOTAL, &g_optin_pair[EPI], "h3_gemm_nvfp4");
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kGemmThreads(EPI));
  cfg.dynamicSmemBytes = GemmPairSmem::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_nvfp4_pair_kernel<EPI>, ta, tb, tsa, tsb, p);
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "h3_gemm_nvfp4: cluster launch: %s", cudaGetErrorString(e));
  return H3_OK;
}

int launch_gemm_pair(int epi, int grid, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa,
                     const CUtensorMap& tsb, const GemmArgs& p, cudaStream_t st) {
  switch (epi) {
    case H3_EPI_STORE: return launch_gemm_pair_t<H3_EPI_STORE>(grid, ta, tb, tsa, tsb, p, st);
    case H3_EPI_GATE_RESID: return launch_gemm_pair_t<H3_EPI_GATE_RESID>(grid, ta, tb, tsa, tsb, p, st);
    case H3_EPI_ACT_BF16: return launch_gemm_pair_t<H3_EPI_ACT_BF16>(grid, ta, tb, tsa, tsb, p, st);
    case H3_EPI_ACT_Q: return launch_gemm_pair_t<H3_EPI_ACT_Q>(grid, ta, tb, tsa, tsb, p, st);
    default: return launch_gemm_pair_t<H3_EPI_STORE_PEERS>(grid, ta, tb, tsa, tsb, p, st);
  }
}

int launch_gemm(int BN, int epi, int grid, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& p,
                cudaStream_t st) {
  switch (epi + 5 * (BN == 256)) {
    case 0: return launch_gemm_t<128, H3_EPI_STORE>(grid, ta, tb, p, st);
    case 1: return launch_gemm_t<128, H3_EPI_GATE_RESID>(grid, ta, tb, p, st);
    case 2: return launch_gemm_t<128, H3_EPI_ACT_BF16>(grid, ta, tb, p, st);
    case 3: return launch_gemm_t<128, H3_EPI_ACT_Q>(grid, ta, tb, p, st);
    case 4: return launch_gemm_t<128, H3_EPI_STORE_PEERS>(grid, ta, tb, p, st);
    case 5: return launch_gemm_t<256, H3_EPI_STORE>(grid, ta, tb, p, st);
    case 6: return launch_gemm_t<256, H3_EPI_GATE_RESID>(grid, ta, tb, p, st);
    case 7: return launch_gemm_t<256, H3_EPI_ACT_BF16>(grid, ta, tb, p, st);
    case 8: return launch_gemm_t<256, H3_EPI_ACT_Q>(grid, ta, tb, p, st);
    default: return launch_gemm_t<256, H3_EPI_STORE_PEERS>(grid, ta, tb, p, st);
  }
}

struct AttnWs {
  size_t q8, k8, vt8, qscale, kscale, kmean, vscale, vinv, ksum, vmax, total;
  int SP, nblk;
};

AttnWs attn_ws(int S, int H) {
  AttnWs w;
  w.SP = (S + 127) / 128 * 128;
  w.nblk = (S + 127) / 128;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align_up(o + bytes, 1024);
    return at;
  };
  w.q8 = take((size_t)H * w.SP * 128);
  w.k8 = take((size_t)H * w.SP * 128);
  w.vt8 = take((size_t)H * w.SP * 128);
  w.qscale = take((size_t)H * w.SP * 4);
  w.kscale = take((size_t)H * (w.SP / 128) * 4);
  w.kmean = take((size_t)H * 128 * 4);
  w.vscale = take((size_t)H * 128 * 4);
  w.vinv = take((size_t)H * 128 * 4);
  w.ksum = take((size_t)w.nblk * H * 128 * 4);
  w.vmax = take((size_t)w.nblk * H * 128 * 4);
  w.total = o;
  return w;
}

}  // namespace

extern "C" {

int h3_version(void) { return H3B200_VERSION; }

int h3_last_error(char* buf, int n) {
  if (buf && n > 0) {
    size_t k = g_err.size() < (size_t)(n - 1) ? g_err.size() : (size_t)(n - 1);
    memcpy(buf, g_err.data(), k);
    buf[k] = 0;
  }
  return (int)g_err.size();
}

int h3_device_status(int* status, int reset) {
  if (!status) return fail(H3_ERR_ARG, "h3_device_status: status is NULL");
  cudaError_t e = cudaMemcpyFromSymbol(status, g_status, sizeof(int));
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "h3_device_status: %s", cudaGetErrorString(e));
  if (reset) {
    int zero = 0;
    e = cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
    if (e != cudaSuccess) return fail(H3_ERR_CUDA, "h3_device_status: %s", cudaGetErrorString(e));
  }
  return H3_OK;
}

}  // extern "C"

namespace {
__global__ void status_publish_kernel(float* dst) { *dst = fmaxf(*dst, (float)*(volatile int*)&g_status); }
}  // namespace

extern "C" {

int h3_status_publish(float* dst, void* stream) {
  if (!dst || !aligned(dst, 4)) return fail(H3_ERR_ARG, "h3_status_publish: dst NULL or misaligned");
  status_publish_kernel<<<1, 1, 0, S_(stream)>>>(dst);
  return check_launch("h3_status_publish");
}

size_t h3_sf_tiled_bytes(int rows, int cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return (size_t)((rows + 127) / 128) * 128 * (size_t)(cols / 16);
}

// ------------------------------------------------------------------------------------------------ peer memory
// Receive buffers of the fused Ulysses exchanges: plain cudaMalloc allocations shared through CUDA IPC handles
// (no multicast object, no NVLS binding), mapped by the other ranks' processes.
int h3_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(H3_ERR_ARG, "h3_peer_alloc: NULL argument or zero bytes");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handle");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "h3_peer_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(H3_ERR_CUDA, "h3_peer_alloc: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return H3_OK;
}

int h3_peer_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(H3_ERR_ARG, "h3_peer_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "h3_peer_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return H3_OK;
}

int h3_peer_close(void* ptr) {
  if (!ptr) return fail(H3_ERR_ARG, "h3_peer_close: NULL pointer");
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "h3_peer_close: %s", cudaGetErrorString(e));
  return H3_OK;
}

namespace {
struct PushArgs {
  const uint4* src[8];
  uint4* dst[8];
  long long n16[8];   // 16-byte words of each copy
};
// blockIdx.y: the copy; grid-stride over its 16-byte words, four loads in flight per thread
__global__ void __launch_bounds__(256) peer_push_kernel(const __grid_constant__ PushArgs a) {
  const int c = blockIdx.y;
  const uint4* __restrict__ src = a.src[c];
  uint4* dst = a.dst[c];
  const long long n = a.n16[c], step = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * step < n; i += 4 * step) {
    const uint4 v0 = src[i], v1 = src[i + step], v2 = src[i + 2 * step], v3 = src[i + 3 * step];
    dst[i] = v0;
    dst[i + step] = v1;
    dst[i + 2 * step] = v2;
    dst[i + 3 * step] = v3;
  }
  for (; i < n; i += step) dst[i] = src[i];
}
}  // namespace

int h3_peer_push(const H3PeerCopy* copies, int n, void* stream) {
  if (!copies || n < 1 || n > 8) return fail(H3_ERR_ARG, "h3_peer_push: need 1..8 copies (n=%d)", n);
  PushArgs a{};
  long long most = 0;
  for (int c = 0; c < n; ++c) {
    if (!copies[c].src || !copies[c].dst || !aligned(copies[c].src, 16) || !aligned(copies[c].dst, 16) ||
        copies[c].bytes % 16)
      return fail(H3_ERR_ARG, "h3_peer_push: copy %d needs 16-byte aligned src/dst and bytes %% 16 == 0", c);
    a.src[c] = reinterpret_cast<const uint4*>(copies[c].src);
    a.dst[c] = reinterpret_cast<uint4*>(copies[c].dst);
    a.n16[c] = (long long)(copies[c].bytes / 16);
    most = a.n16[c] > most ? a.n16[c] : most;
  }
  if (most == 0) return H3_OK;
  // about one 128-thread block (6 K registers) per SM over all n copies: one fits beside a persistent GEMM CTA on
  // its SM, so a push issued on a side stream runs while the GEMM computes the next rows
  long long blocks = (most + 511) / 512;
  const long long cap = num_sms() / n > 0 ? num_sms() / n : 1;   // per copy
  if (blocks > cap) blocks = cap;
  peer_push_kernel<<<dim3((unsigned)blocks, n), 128, 0, S_(stream)>>>(a);
  return check_launch("h3_peer_push");
}

int h3_peer_copy(const H3PeerCopy* copies, int n, void* stream) {
  if (!copies || n < 0) return fail(H3_ERR_ARG, "h3_peer_copy: NULL copies or n < 0");
  for (int c = 0; c < n; ++c) {
    if (!copies[c].bytes) continue;
    if (!copies[c].src || !copies[c].dst) return fail(H3_ERR_ARG, "h3_peer_copy: copy %d has a NULL pointer", c);
    cudaError_t e = cudaMemcpyAsync(copies[c].dst, copies[c].src, copies[c].bytes, cudaMemcpyDeviceToDevice,
                                    S_(stream));
    if (e != cudaSuccess) return fail(H3_ERR_CUDA, "h3_peer_copy: copy %d: %s", c, cudaGetErrorString(e));
  }
  return H3_OK;
}

int h3_peer_free(void* ptr) {
  if (!ptr) return fail(H3_ERR_ARG, "h3_peer_free: NULL pointer");
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "h3_peer_free: %s", cudaGetErrorString(e));
  return H3_OK;
}

// ------------------------------------------------------------------------------------------------ scales
int h3_scales_begin(H3ScaleSlot* slots, int n, int delayed, int* clipped, void* stream) {
  if (!slots || n <= 0) return fail(H3_ERR_ARG, "h3_scales_begin: slots NULL or n <= 0");
  scales_begin_kernel<<<(n + 127) / 128, 128, 0, S_(stream)>>>(slots, n, delayed, clipped);
  return check_launch("h3_scales_begin");
}

int h3_scales_dynamic(H3ScaleSlot* slot, void* stream) {
  if (!slot) return fail(H3_ERR_ARG, "h3_scales_dynamic: slot is NULL");
  act_from_amax_kernel<<<1, 1, 0, S_(stream)>>>(slot);
  return check_launch("h3_scales_dynamic");
}

int h3_absmax_bf16(const void* x, long long ldx, int R, int K, float* out, void* stream) {
  if (!x || !out) return fail(H3_ERR_ARG, "h3_absmax_bf16: NULL pointer");
  if (R <= 0 || K <= 0 || K % 8 || ldx % 8 || !aligned(x, 16))
    return fail(H3_ERR_SHAPE, "h3_absmax_bf16: need K %% 8 == 0, ldx %% 8 == 0, 16-byte aligned x");
  long long n = (long long)R * (K / 8);
  int blocks = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  absmax_kernel<<<blocks, 256, 0, S_(stream)>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, R, K, out);
  return check_launch("h3_absmax_bf16");
}

// ------------------------------------------------------------------------------------------------ elementwise
int h3_norm_mod(const void* x, int ldx, const float* w, const float* mod, const int* idx, int S, int D, int part,
                float eps, void* out, int ldo, uint8_t* codes, uint8_t* sf, int sf_tiled, H3ScaleSlot* slot,
                void* stream) {
  if (!x || !w || !mod || !idx) return fail(H3_ERR_ARG, "h3_norm_mod: NULL input");
  if (!out && !codes && !slot) return fail(H3_ERR_ARG, "h3_norm_mod: no output requested");
  if (codes && (!sf || !slot)) return fail(H3_ERR_ARG, "h3_norm_mod: quantised output needs sf and slot");
  if (part != 0 && part != 1) return fail(H3_ERR_ARG, "h3_norm_mod: part must be 0 or 1");
  if (S <= 0 || D <= 0 || D % 16 || D > 6144 || ldx % 8 || (out && ldo % 8))
    return fail(H3_ERR_SHAPE, "h3_norm_mod: need D %% 16 == 0, D <= 6144, row strides %% 8 == 0 (D=%d)", D);
  if (!aligned(x, 16) || (out && !aligned(out, 16)) || (codes && !aligned(codes, 4)) || !aligned(w, 16) ||
      !aligned(mod, 16))
    return fail(H3_ERR_ARG, "h3_norm_mod: misaligned pointer");
  NormModArgs a{reinterpret_cast<const __nv_bfloat16*>(x), ldx, w, mod, idx, S, D, part, eps,
                reinterpret_cast<__nv_bfloat16*>(out), ldo, codes, sf, sf_tiled, slot};
  const int rows_per_block = 8;
  const dim3 grid((S + rows_per_block - 1) / rows_per_block), block(32 * rows_per_block);
  norm_mod_kernel<<<grid, block, 0, S_(stream)>>>(a);
  return check_launch("h3_norm_mod");
}

int h3_nvfp4_quant(const void* x, long long ldx, int cblk, long long blk_stride, int R, int K, const float* g_dev,
                   float g, uint8_t* codes, uint8_t* sf, int sf_tiled, float* amax, void* stream) {
  if (!x || !codes || !sf) return fail(H3_ERR_ARG, "h3_nvfp4_quant: NULL pointer");
  if (R <= 0 || K <= 0 || K % 16 || cblk <= 0 || cblk % 16 || ldx % 8 || blk_stride % 8)
    return fail(H3_ERR_SHAPE, "h3_nvfp4_quant: need K, cblk %% 16 == 0 and strides %% 8 == 0");
  if (!g_dev && !(g > 0.f)) return fail(H3_ERR_ARG, "h3_nvfp4_quant: global scale must be > 0");
  if (!aligned(x, 16) || !aligned(codes, 8)) return fail(H3_ERR_ARG, "h3_nvfp4_quant: misaligned pointer");
  QuantArgs a{reinterpret_cast<const __nv_bfloat16*>(x), ldx, cblk, blk_stride, R, K, g_dev, g, codes, sf, sf_tiled,
              amax};
  long long n = (long long)R * (K / 16);
  nvfp4_quant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, S_(stream)>>>(a);
  return check_launch("h3_nvfp4_quant");
}

int h3_gate_add(void* x, int ldx, const void* y, int ldy, const float* mod, const int* idx, int S, int D, int part,
                void* stream) {
  if (!x || !y || !mod || !idx) return fail(H3_ERR_ARG, "h3_gate_add: NULL pointer");
  if (S <= 0 || D <= 0 || D % 8 || ldx % 8 || ldy % 8) return fail(H3_ERR_SHAPE, "h3_gate_add: need D %% 8 == 0");
  if (part != 0 && part != 1) return fail(H3_ERR_ARG, "h3_gate_add: part must be 0 or 1");
  long long n = (long long)S * (D / 8);
  int blocks = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  gate_add_kernel<<<blocks, 256, 0, S_(stream)>>>(reinterpret_cast<__nv_bfloat16*>(x), ldx,
                                                  reinterpret_cast<const __nv_bfloat16*>(y), ldy, mod, idx, S, D,
                                                  part);
  return check_launch("h3_gate_add");
}

int h3_act(const void* u, int ldu, void* out, int ldo, int M, int F, int act_kind, float* amax, void* stream) {
  if (!u || !out) return fail(H3_ERR_ARG, "h3_act: NULL pointer");
  if (M <= 0 || F <= 0 || F % 8 || ldu % 8 || ldo % 8) return fail(H3_ERR_SHAPE, "h3_act: need F %% 8 == 0");
  if (act_kind != 0 && act_kind != 1) return fail(H3_ERR_ARG, "h3_act: act_kind must be 0 or 1");
  long long n = (long long)M * (F / 8);
  int blocks = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  act_kernel<<<blocks, 256, 0, S_(stream)>>>(reinterpret_cast<const __nv_bfloat16*>(u), ldu,
                                             reinterpret_cast<__nv_bfloat16*>(out), ldo, M, F, act_kind, amax);
  return check_launch("h3_act");
}

int h3_modulation(const float* t_emb, int M, int t_dim, const float* ada_w, const float* ada_b, int J, float* mod,
                  void* stream) {
  if (!t_emb || !ada_w || !ada_b || !mod) return fail(H3_ERR_ARG, "h3_modulation: NULL pointer");
  if (M <= 0 || t_dim <= 0 || J <= 0) return fail(H3_ERR_SHAPE, "h3_modulation: bad sizes");
  long long n = (long long)M * J;
  modulation_kernel<<<(unsigned)((n + 255) / 256), 256, 0, S_(stream)>>>(t_emb, M, t_dim, ada_w, ada_b, J, mod);
  return check_launch("h3_modulation");
}

// ------------------------------------------------------------------------------------------------ GEMM
int h3_gemm_nvfp4(const uint8_t* a_codes, const uint8_t* a_sf, const H3ScaleSlot* a_slot, const uint8_t* b_codes,
                  const uint8_t* b_sf, float g_b, const float* bias, int M, int N, int K, const H3Epilogue* epi,
                  void* stream) {
  if (!a_codes || !a_sf || !a_slot || !b_codes || !b_sf || !epi) return fail(H3_ERR_ARG, "h3_gemm_nvfp4: NULL pointer");
  if (M <= 0 || N <= 0 || K <= 0 || K % 256 || N % 128)
    return fail(H3_ERR_SHAPE, "h3_gemm_nvfp4: need K %% 256 == 0 and N %% 128 == 0 (M=%d N=%d K=%d)", M, N, K);
  if (!aligned(a_codes, 16) || !aligned(b_codes, 16) || !aligned(a_sf, 16) || !aligned(b_sf, 16))
    return fail(H3_ERR_ARG, "h3_gemm_nvfp4: codes and scales must be 16-byte aligned");
  GemmArgs p{};
  p.sfa = a_sf;
  p.sfb = b_sf;
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_slot = a_slot;
  p.g_b = g_b;
  p.bias = bias;
  p.epi = epi->kind;
  p.out = reinterpret_cast<__nv_bfloat16*>(epi->out);
  p.ldo = epi->ldo;
  p.x = reinterpret_cast<__nv_bfloat16*>(epi->x);
  p.ldx = epi->ldx;
  p.mod = epi->mod;
  p.idx = epi->idx;
  p.gate_part = epi->gate_part;
  p.act_kind = epi->act_kind;
  p.qcodes = epi->qcodes;
  p.qsf = epi->qsf;
  p.q_slot = epi->q_slot;
  switch (epi->kind) {
    case H3_EPI_STORE:
      if (!p.out || p.ldo % 8 || !aligned(p.out, 16)) return fail(H3_ERR_ARG, "h3_gemm_nvfp4: STORE needs out");
      break;
    case H3_EPI_STORE_PEERS:
      if (epi->ranks < 1 || epi->ranks > 8 || epi->rank < 0 || epi->rank >= epi->ranks || N % (384 * epi->ranks))
        return fail(H3_ERR_ARG, "h3_gemm_nvfp4: STORE_PEERS needs 1 <= ranks <= 8, 0 <= rank < ranks and N a "
                                "multiple of 3 * 128 * ranks (ranks=%d rank=%d N=%d)", epi->ranks, epi->rank, N);
      for (int r = 0; r < epi->ranks; ++r) {
        if (!epi->peer[r] || !aligned(epi->peer[r], 16))
          return fail(H3_ERR_ARG, "h3_gemm_nvfp4: STORE_PEERS peer[%d] NULL or not 16-byte aligned", r);
        p.peer[r] = reinterpret_cast<unsigned long long>(epi->peer[r]);
      }
      p.ranks = epi->ranks;
      p.rank = epi->rank;
      break;
    case H3_EPI_GATE_RESID:
      if (!p.x || !p.mod || !p.idx || p.ldx % 8 || !aligned(p.x, 16) || (p.gate_part != 0 && p.gate_part != 1))
        return fail(H3_ERR_ARG, "h3_gemm_nvfp4: GATE_RESID needs x, mod, idx, gate_part");
      break;
    case H3_EPI_ACT_BF16:
    case H3_EPI_ACT_Q:
      if (p.act_kind != 0 && p.act_kind != 1) return fail(H3_ERR_ARG, "h3_gemm_nvfp4: act_kind must be 0 or 1");
      if (epi->kind == H3_EPI_ACT_BF16 && !p.out) return fail(H3_ERR_ARG, "h3_gemm_nvfp4: ACT_BF16 needs out");
      if (epi->kind == H3_EPI_ACT_Q && (!p.qcodes || !p.qsf || !p.q_slot))
        return fail(H3_ERR_ARG, "h3_gemm_nvfp4: ACT_Q needs qcodes, qsf, q_slot");
      if (p.out && (p.ldo % 8 || !aligned(p.out, 16))) return fail(H3_ERR_ARG, "h3_gemm_nvfp4: misaligned out");
      break;
    default:
      return fail(H3_ERR_ARG, "h3_gemm_nvfp4: unknown epilogue %d", epi->kind);
  }
  CUtensorMap ta, tb;
  int rc = make_map_u8(&ta, a_codes, K / 2, M, K / 2, 128, 128, "h3_gemm_nvfp4(A)");
  if (rc) return rc;
  if (H3_GEMM_PAIR && N % 256 == 0 && num_sms() >= 2) {   // CTA pairs over 256 x 256 tiles
    CUtensorMap tsa, tsb;
    if ((rc = make_map_u8(&tb, b_codes, K / 2, N, K / 2, 128, 128, "h3_gemm_nvfp4(B)"))) return rc;
    if ((rc = make_map_sf_rows(&tsa, a_sf, (uint64_t)((M + 127) / 128) * (K / 256), "h3_gemm_nvfp4(A scales)")))
      return rc;
    if ((rc = make_map_sf_rows(&tsb, b_sf, (uint64_t)(N / 128) * (K / 256), "h3_gemm_nvfp4(B scales)"))) return rc;
    const int tiles = (N / 256) * ((M + 255) / 256);
    const int pairs = tiles < num_sms() / 2 ? tiles : num_sms() / 2;
    if ((rc = launch_gemm_pair(epi->kind, 2 * pairs, ta, tb, tsa, tsb, p, S_(stream)))) return rc;
    return check_launch("h3_gemm_nvfp4");
  }
  const int BN = (N % 256 == 0) ? 256 : 128;
  rc = make_map_u8(&tb, b_codes, K / 2, N, K / 2, 128, BN, "h3_gemm_nvfp4(B)");
  if (rc) return rc;
  const int tiles = (N / BN) * ((M + 127) / 128);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  rc = launch_gemm(BN, epi->kind, grid, ta, tb, p, S_(stream));
  if (rc) return rc;
  return check_launch("h3_gemm_nvfp4");
}

// ------------------------------------------------------------------------------------------------ attention
int h3_qknorm_rope(void* q, void* k, long long ld, int S, int H, int rot, const float* qw, const float* kw,
                   const float* rope, float eps, void* stream) {
  if (!q || !k || !qw || !kw || (rot > 0 && !rope)) return fail(H3_ERR_ARG, "h3_qknorm_rope: NULL pointer");
  if (S <= 0 || H <= 0 || rot < 0 || rot > 128 || rot % 8 || ld % 4)
    return fail(H3_ERR_SHAPE, "h3_qknorm_rope: need rot %% 8 == 0, rot <= 128, ld %% 4 == 0");
  if (!aligned(q, 8) || !aligned(k, 8) || (rope && !aligned(rope, 16)))
    return fail(H3_ERR_ARG, "h3_qknorm_rope: misaligned pointer");
  QkNormArgs a{reinterpret_cast<__nv_bfloat16*>(q), reinterpret_cast<__nv_bfloat16*>(k), ld, S, H, rot, qw, kw, rope,
               eps};
  qknorm_rope_kernel<<<(unsigned)((S + 7) / 8), 256, 0, S_(stream)>>>(a);
  return check_launch("h3_qknorm_rope");
}

size_t h3_attn_workspace_bytes(int S, int H) {
  if (S <= 0 || H <= 0) return 0;
  return attn_ws(S, H).total;
}

namespace {
// Prepare (K mean / V max, FP8 quantisation) and the attention kernel, dense (kv_ptr NULL) or block-sparse.
struct PeerOut {   // h3_attn_fp8_peers: output rows to the ranks that own the tokens
  void* const* peer;
  int ranks, rank;
};

int attn_run(const char* who, const void* q, const void* k, const void* v, long long ld, long long hstride, int S,
             int H, const int* kv_ptr, const int* kv_idx, void* out, long long ldo, void* workspace,
             size_t workspace_bytes, void* stream, const PeerOut* po = nullptr) {
  if (po) {
    if (!po->peer || po->ranks < 1 || po->ranks > 8 || po->rank < 0 || po->rank >= po->ranks || S % po->ranks)
      return fail(H3_ERR_ARG, "%s: need 1 <= ranks <= 8, 0 <= rank < ranks, S %% ranks == 0 (S=%d ranks=%d rank=%d)",
                  who, S, po->ranks, po->rank);
    for (int r = 0; r < po->ranks; ++r)
      if (!po->peer[r] || !aligned(po->peer[r], 16)) return fail(H3_ERR_ARG, "%s: peer[%d] NULL or misaligned", who, r);
    if (ldo < (long long)H * 128) return fail(H3_ERR_ARG, "%s: receive rows of %lld < H * 128 elements", who, ldo);
    out = po->peer[po->rank];
  }
  if (!q || !k || !v || !out || !workspace) return fail(H3_ERR_ARG, "%s: NULL pointer", who);
  if (S <= 0 || H <= 0 || ld % 8 || hstride % 8 || ldo % 8)
    return fail(H3_ERR_SHAPE, "%s: need strides %% 8 == 0", who);
  constexpr int kMaxS = AttnSmem<2>::MAX_KBLK * 128;
  static_assert(AttnSmem<1>::MAX_KBLK == AttnSmem<2>::MAX_KBLK, "one sequence limit");
  if (S > kMaxS || H > 65535)
    return fail(H3_ERR_SHAPE, "%s: S=%d, H=%d beyond the supported S <= %d, H <= 65535", who, S, H, kMaxS);
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16) || !aligned(workspace, 1024))
    return fail(H3_ERR_ARG, "%s: q/k/v/out 16-byte and workspace 1024-byte alignment required", who);
  AttnWs w = attn_ws(S, H);
  if (workspace_bytes < w.total)
    return fail(H3_ERR_ARG, "%s: workspace %zu bytes < %zu", who, workspace_bytes, w.total);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  uint8_t* q8 = ws + w.q8;
  uint8_t* k8 = ws + w.k8;
  uint8_t* vt8 = ws + w.vt8;
  float* qscale = reinterpret_cast<float*>(ws + w.qscale);
  float* kscale = reinterpret_cast<float*>(ws + w.kscale);
  float* kmean = reinterpret_cast<float*>(ws + w.kmean);
  float* vscale = reinterpret_cast<float*>(ws + w.vscale);
  float* vinv = reinterpret_cast<float*>(ws + w.vinv);
  float* ksum = reinterpret_cast<float*>(ws + w.ksum);
  float* vmax = reinterpret_cast<float*>(ws + w.vmax);
  AttnView view{reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
                reinterpret_cast<const __nv_bfloat16*>(v), ld, hstride};
  cudaStream_t st = S_(stream);
  attn_stats_kernel<<<dim3(w.nblk, H), 128, 0, st>>>(view, S, H, ksum, vmax);
  int rc = check_launch(who);
  if (rc) return rc;
  attn_stats_reduce_kernel<<<(H * 128 + 127) / 128, 128, 0, st>>>(ksum, vmax, w.nblk, S, H, kmean, vscale, vinv);
  if ((rc = check_launch(who))) return rc;
  attn_quant_kernel<<<dim3(w.SP / 128, H), 128, 0, st>>>(view, S, w.SP, H, kmean, vinv, q8, qscale, k8, kscale, vt8);
  if ((rc = check_launch(who))) return rc;
  CUtensorMap tq, tk, tv;
  if ((rc = make_map_u8(&tq, q8, 128, (uint64_t)H * w.SP, 128, 128, 128, who))) return rc;
  if ((rc = make_map_u8(&tk, k8, 128, (uint64_t)H * w.SP, 128, 128, 128, who))) return rc;
  if ((rc = make_map_u8(&tv, vt8, w.SP, (uint64_t)H * 128, w.SP, 128, 128, who))) return rc;
  AttnArgs p{qscale, kscale, vscale, reinterpret_cast<__nv_bfloat16*>(out), ldo, S, w.SP, H, kv_ptr, kv_idx};
  if (po) {
    for (int r = 0; r < po->ranks; ++r) p.peer[r] = reinterpret_cast<unsigned long long>(po->peer[r]);
    p.ranks = po->ranks;
    p.rank = po->rank;
    p.n_local = S / po->ranks;
  }
  if (kv_ptr) {   // block-sparse: one query tile per CTA (each has its own KV list), two CTAs per SM
    if ((rc = smem_optin(attn_fp8_kernel<1>, AttnSmem<1>::TOTAL, &g_optin_attn[0], who))) return rc;
    attn_fp8_kernel<1><<<dim3((S + kQTile - 1) / kQTile, H), attn_threads(1), AttnSmem<1>::TOTAL, st>>>(tq, tk, tv, p);
  } else {
    if ((rc = smem_optin(attn_fp8_kernel<2>, AttnSmem<2>::TOTAL, &g_optin_attn[1], who))) return rc;
    attn_fp8_kernel<2><<<dim3((S + 2 * kQTile - 1) / (2 * kQTile), H), attn_threads(2), AttnSmem<2>::TOTAL, st>>>(
        tq, tk, tv, p);
  }
  return check_launch(who);
}
}  // namespace

int h3_attn_fp8(const void* q, const void* k, const void* v, long long ld, long long hstride, int S, int H, void* out,
                long long ldo, void* workspace, size_t workspace_bytes, void* stream) {
  return attn_run("h3_attn_fp8", q, k, v, ld, hstride, S, H, nullptr, nullptr, out, ldo, workspace, workspace_bytes,
                  stream);
}

int h3_attn_fp8_peers(const void* q, const void* k, const void* v, long long ld, long long hstride, int S, int H,
                      const int* kv_ptr, const int* kv_idx, void* const* peer, int ranks, int rank, long long ldo,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if ((kv_ptr == nullptr) != (kv_idx == nullptr)) return fail(H3_ERR_ARG, "h3_attn_fp8_peers: half a tile list");
  if (kv_ptr && (!aligned(kv_ptr, 4) || !aligned(kv_idx, 4)))
    return fail(H3_ERR_ARG, "h3_attn_fp8_peers: misaligned tile list");
  const PeerOut po{peer, ranks, rank};
  return attn_run("h3_attn_fp8_peers", q, k, v, ld, hstride, S, H, kv_ptr, kv_idx, nullptr, ldo, workspace,
                  workspace_bytes, stream, &po);
}

int h3_attn_fp8_sparse(const void* q, const void* k, const void* v, long long ld, long long hstride, int S, int H,
                       const int* kv_ptr, const int* kv_idx, void* out, long long ldo, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (!kv_ptr || !kv_idx) return fail(H3_ERR_ARG, "h3_attn_fp8_sparse: NULL tile list");
  if (!aligned(kv_ptr, 4) || !aligned(kv_idx, 4)) return fail(H3_ERR_ARG, "h3_attn_fp8_sparse: misaligned tile list");
  return attn_run("h3_attn_fp8_sparse", q, k, v, ld, hstride, S, H, kv_ptr, kv_idx, out, ldo, workspace,
                  workspace_bytes, stream);
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------ no-alloc attention
// Scratch of h3_attn_fp8_noalloc: one file-scope device array of kNoAllocScratchBytes.  Every GPU that loads this
// library holds it until the process exits.  Host code must not pass the symbol itself to a kernel (on the host it
// names a stand-in, not device memory): its device address comes from cudaGetSymbolAddress, looked up once per
// device with that device current.
constexpr size_t kNoAllocScratchBytes = 64ull << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
// The array's device address is looked up once per (device, CUDA context) and cached with the context it belongs to:
// a caller that resets the device or switches to another context on it gets the module loaded again, possibly at a
// different address, and the lookup is then repeated for that context.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

struct NoAllocSlot {
  CUcontext ctx;
  void* ptr;
};
std::mutex g_noalloc_mu;
NoAllocSlot g_noalloc[64] = {};

int noalloc_scratch(const char* who, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(H3_ERR_CUDA, "%s: cudaGetDevice: %s", who, cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(H3_ERR_ARG, "%s: device %d out of range", who, dev);
  CtxGetCurrentFn get = ctx_get_current_fn();
  if (!get) return fail(H3_ERR_CUDA, "%s: cuCtxGetCurrent unavailable from the driver", who);
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) return fail(H3_ERR_CUDA, "%s: cuCtxGetCurrent failed", who);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocSlot& slot = g_noalloc[dev];
  if (ctx && slot.ptr && slot.ctx == ctx) {
    *out = slot.ptr;
    return H3_OK;
  }
  // first call in this context (or none current yet: the runtime's lookup makes the device's primary context current)
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p) return fail(H3_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
  if (get(&ctx) != CUDA_SUCCESS || !ctx) return fail(H3_ERR_CUDA, "%s: no current CUDA context after set-up", who);
  slot.ctx = ctx;
  slot.ptr = p;
  *out = p;
  return H3_OK;
}
}  // namespace

extern "C" {

int h3_attn_fp8_noalloc(const void* q, const void* k, const void* v, long long ld, long long hstride, int S, int H,
                        void* out, long long ldo, void* stream) {
  const char* who = "h3_attn_fp8_noalloc";
  if (S <= 0 || H <= 0) return fail(H3_ERR_SHAPE, "%s: S and H must be positive", who);
  const size_t need = h3_attn_workspace_bytes(S, H);
  if (need + 1024 > kNoAllocScratchBytes)
    return fail(H3_ERR_SHAPE,
                "%s: S=%d, H=%d needs %zu bytes of scratch, beyond the fixed %zu-byte array; use h3_attn_fp8 with a "
                "caller-provided workspace",
                who, S, H, need, kNoAllocScratchBytes - 1024);
  void* base = nullptr;
  int rc = noalloc_scratch(who, &base);
  if (rc) return rc;
  // the workspace layout wants a 1024-byte aligned start; the array is 256-aligned, so step to the next 1024
  uint8_t* ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(base) + 1023) & ~uintptr_t(1023));
  return attn_run(who, q, k, v, ld, hstride, S, H, nullptr, nullptr, out, ldo, ws, kNoAllocScratchBytes - 1024,
                  stream);
}

}  // extern "C"
