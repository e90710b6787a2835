// Attention half of the block for sm_100a: per-head QK-RMSNorm + split-half RoPE (the call
// ck.rms_rope_split_half_ at tfvideo/minimax_h3.py:296-298), the FP8 prepare (sequence statistics, Q/K/V -> e4m3 with
// fp32 scales; tfvideo/fp4attn.py:82-147) and the FP8 flash attention itself (tfvideo/fp4attn.py:170-238) on
// tcgen05: QK^T and PV as kind::f8f6f4 MMAs with S, P and O in TMEM, K/V tiles streamed by TMA, online softmax in
// registers.
//
// Recipe (per head): K is smoothed by its per-channel mean over the sequence; Q carries log2(e)/sqrt(Dh) and one fp32
// scale per row (rowmax / 448); K one fp32 scale per 128-key block (blockmax / 448); V one scale per channel
// (vmax / 448), applied in the epilogue; P = exp2(s - m + c) is written to TMEM as e4m3 with c = log2(448) - tau, so
// P <= 448 while the running max m lags the true max by at most tau (the max is only raised, and O rescaled, when a
// row's max grows by more than tau).
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "h3b200.h"

namespace h3 {

constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------------------------------------------------ qk norm + rope
// One warp per (token, q|k, head) row of Dh = 128; lane l owns dims 4l..4l+3.  y = x / sqrt(mean(x^2) + eps) * w;
// pair i < rot/2 couples dims i and i + rot/2 through the token's 2x2 matrix rope[s, i] (o_i = f00 y_i + f01 y_j,
// o_j = f10 y_i + f11 y_j); dims >= rot pass through.  In place on the bf16 rows.
struct QkNormArgs {
  __nv_bfloat16* q;      // element (s, h, d) at q + s * ld + h * 128 + d
  __nv_bfloat16* k;
  long long ld;
  int S, H, rot;
  const float* qw;
  const float* kw;
  const float* rope;     // fp32 [S, rot/2, 2, 2]
  float eps;
};

// One warp per token: its RoPE matrices are loaded once into registers (lane l's dims 4l..4l+3 need pairs 4l..4l+3
// when they lie in the first half of the rotated span, 4l - rot/2.. in the second) and applied to the token's 2H head
// rows, two rows in flight at a time.
__device__ __forceinline__ void qk_row(__nv_bfloat16* row, const float* w, const float (&f)[4][4], int lane, int half,
                                       int rot, int src, float eps) {
  uint2 u = *reinterpret_cast<const uint2*>(row + lane * 4);
  float x[4] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y)};
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
#pragma unroll
  for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), eps)));
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) y[e] = __fmul_rn(__fmul_rn(x[e], r), w[e]);
  float pv[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) pv[e] = __shfl_sync(0xffffffffu, y[e], src);
  float o[4];
  const int d0 = lane * 4;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (d0 < half)
      o[e] = __fadd_rn(__fmul_rn(f[e][0], y[e]), __fmul_rn(f[e][1], pv[e]));
    else if (d0 < rot)
      o[e] = __fadd_rn(__fmul_rn(f[e][2], pv[e]), __fmul_rn(f[e][3], y[e]));
    else
      o[e] = y[e];
  }
  *reinterpret_cast<uint2*>(row + lane * 4) = make_uint2(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]));
}

__global__ void __launch_bounds__(256) qknorm_rope_kernel(QkNormArgs a) {
  const int lane = threadIdx.x & 31;
  const int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (s >= a.S) return;
  const int half = a.rot >> 1, hq = half >> 2;
  const int d0 = lane * 4;
  int src = lane;
  if (d0 < half) src = lane + hq;
  else if (d0 < a.rot) src = lane - hq;
  float f[4][4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = d0 + e;
    const int pair = d < half ? d : d - half;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (d < a.rot) v = *reinterpret_cast<const float4*>(a.rope + ((size_t)s * half + pair) * 4);
    f[e][0] = v.x;
    f[e][1] = v.y;
    f[e][2] = v.z;
    f[e][3] = v.w;
  }
  float qw[4], kw[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    qw[e] = a.qw[d0 + e];
    kw[e] = a.kw[d0 + e];
  }
  __nv_bfloat16* qrow = a.q + (long long)s * a.ld;
  __nv_bfloat16* krow = a.k + (long long)s * a.ld;
#pragma unroll 2
  for (int h = 0; h < a.H; ++h) {
    qk_row(qrow + h * 128, qw, f, lane, half, a.rot, src, a.eps);
    qk_row(krow + h * 128, kw, f, lane, half, a.rot, src, a.eps);
  }
}

// ------------------------------------------------------------------------------------------------ prepare
// Views of q, k, v: element (t, h, d) at base + t * ld + h * hstride + d (covers the [S, 3 H Dh] qkv rows and the
// [S, H/P, Dh] Ulysses receive buffers).
struct AttnView {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long long ld;
  long long hstride;
};

// Per (128-token block, head): partial channel sums of k and channel maxima of |v| -> part[blk][h][d] (sum) and
// part[nblk][H][128] + ... (max) in the workspace; fixed order, so the statistics are deterministic.
__global__ void __launch_bounds__(128) attn_stats_kernel(AttnView a, int S, int H, float* ksum_part, float* vmax_part) {
  // thread (g, c8): channels 8 c8 .. 8 c8 + 7 over tokens t0 + g, t0 + g + 8, ... (16-byte loads); the 8 token groups
  // are combined in a fixed order through shared memory
  __shared__ float red_s[8][128], red_m[8][128];
  const int blk = blockIdx.x, h = blockIdx.y;
  const int c8 = threadIdx.x & 15, g = threadIdx.x >> 4;
  const int t0 = blk * 128, t1 = min(S, t0 + 128);
  float ks[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, vm[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int t = t0 + g; t < t1; t += 8) {
    const long long off = (long long)t * a.ld + (long long)h * a.hstride + c8 * 8;
    const uint4 ku = *reinterpret_cast<const uint4*>(a.k + off);
    const uint4 vu = *reinterpret_cast<const uint4*>(a.v + off);
    const uint32_t kw[4] = {ku.x, ku.y, ku.z, ku.w}, vw[4] = {vu.x, vu.y, vu.z, vu.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ks[2 * j] = __fadd_rn(ks[2 * j], bf16_lo(kw[j]));
      ks[2 * j + 1] = __fadd_rn(ks[2 * j + 1], bf16_hi(kw[j]));
      vm[2 * j] = fmaxf(vm[2 * j], fabsf(bf16_lo(vw[j])));
      vm[2 * j + 1] = fmaxf(vm[2 * j + 1], fabsf(bf16_hi(vw[j])));
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    red_s[g][c8 * 8 + e] = ks[e];
    red_m[g][c8 * 8 + e] = vm[e];
  }
  __syncthreads();
  const int d = threadIdx.x;
  float sum = 0.f, mx = 0.f;
#pragma unroll
  for (int gg = 0; gg < 8; ++gg) {
    sum = __fadd_rn(sum, red_s[gg][d]);
    mx = fmaxf(mx, red_m[gg][d]);
  }
  ksum_part[((size_t)blk * H + h) * 128 + d] = sum;
  vmax_part[((size_t)blk * H + h) * 128 + d] = mx;
}

// kmean[h][d] = sum over blocks / S; vscale[h][d] = vmax / 448 (the epilogue's per-channel factor), vinv = 448 / vmax.
__global__ void attn_stats_reduce_kernel(const float* ksum_part, const float* vmax_part, int nblk, int S, int H,
                                         float* kmean, float* vscale, float* vinv) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= H * 128) return;
  float ks = 0.f, vm = 0.f;
  for (int b = 0; b < nblk; ++b) {
    ks = __fadd_rn(ks, ksum_part[(size_t)b * H * 128 + i]);
    vm = fmaxf(vm, vmax_part[(size_t)b * H * 128 + i]);
  }
  kmean[i] = __fdiv_rn(ks, (float)S);
  vm = fmaxf(vm, 1e-30f);
  vscale[i] = __fdiv_rn(vm, 448.0f);
  vinv[i] = __fdiv_rn(448.0f, vm);
}

// Per (128-token block, head), thread = token: Q row -> e4m3 [H][SP][128] + fp32 scale [H][SP]; K row (smoothed) ->
// e4m3 with one scale per block [H][SP/128]; V -> e4m3 transposed [H][128][SP] (keys contiguous, the K-major B operand
// of PV).  Rows t >= S are written as zeros.
__global__ void __launch_bounds__(128) attn_quant_kernel(AttnView a, int S, int SP, int H, const float* kmean,
                                                         const float* vinv, uint8_t* q8, float* qscale, uint8_t* k8,
                                                         float* kscale, uint8_t* vt8) {
  __shared__ float red[4];
  const int blk = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int t = blk * 128 + tid;
  const bool live = t < S;
  const long long base = (long long)t * a.ld + (long long)h * a.hstride;
  const float qmul = kLog2e / sqrtf(128.0f);
  uint32_t outw[32];
  // ---- Q
  {
    float amax = 0.f;
    float x[128];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 u = live ? *reinterpret_cast<const uint4*>(a.q + base + c * 8) : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[c * 8 + 2 * j] = __fmul_rn(bf16_lo(w[j]), qmul);
        x[c * 8 + 2 * j + 1] = __fmul_rn(bf16_hi(w[j]), qmul);
      }
    }
#pragma unroll
    for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const float qr = __fdiv_rn(fmaxf(amax, 1e-30f), 448.0f);
    const float inv = __fdiv_rn(1.0f, qr);
#pragma unroll
    for (int w = 0; w < 32; ++w)
      outw[w] = e4m3x2(__fmul_rn(x[4 * w], inv), __fmul_rn(x[4 * w + 1], inv)) |
                (e4m3x2(__fmul_rn(x[4 * w + 2], inv), __fmul_rn(x[4 * w + 3], inv)) << 16);
    uint4* dst = reinterpret_cast<uint4*>(q8 + ((size_t)h * SP + t) * 128);
#pragma unroll
    for (int c = 0; c < 8; ++c) dst[c] = make_uint4(outw[4 * c], outw[4 * c + 1], outw[4 * c + 2], outw[4 * c + 3]);
    qscale[(size_t)h * SP + t] = qr;   // tiny but finite for padded rows: no NaN from masked keys
  }
  // ---- K (smoothed, one scale per 128-key block)
  {
    float x[128];
    float amax = 0.f;
    const float* km = kmean + h * 128;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 u = live ? *reinterpret_cast<const uint4*>(a.k + base + c * 8) : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = c * 8 + 2 * j;
        x[d] = live ? __fsub_rn(bf16_lo(w[j]), km[d]) : 0.f;
        x[d + 1] = live ? __fsub_rn(bf16_hi(w[j]), km[d + 1]) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(x[i]));
    amax = warp_max(amax);
    if ((tid & 31) == 0) red[tid >> 5] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float kr = __fdiv_rn(fmaxf(amax, 1e-30f), 448.0f);
    const float inv = __fdiv_rn(1.0f, kr);
#pragma unroll
    for (int w = 0; w < 32; ++w)
      outw[w] = e4m3x2(__fmul_rn(x[4 * w], inv), __fmul_rn(x[4 * w + 1], inv)) |
                (e4m3x2(__fmul_rn(x[4 * w + 2], inv), __fmul_rn(x[4 * w + 3], inv)) << 16);
    uint4* dst = reinterpret_cast<uint4*>(k8 + ((size_t)h * SP + t) * 128);
#pragma unroll
    for (int c = 0; c < 8; ++c) dst[c] = make_uint4(outw[4 * c], outw[4 * c + 1], outw[4 * c + 2], outw[4 * c + 3]);
    if (tid == 0) kscale[(size_t)h * (SP / 128) + blk] = kr;
  }
  // ---- V (per channel), transposed through shared memory: thread t writes column t of the [128 d][128 t] tile,
  // then each thread stores one row d with 16-byte writes
  {
    __shared__ uint32_t vt[128][33];   // [d][t / 4] words, padded
    const float* vi = vinv + h * 128;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 u = live ? *reinterpret_cast<const uint4*>(a.v + base + c * 8) : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = c * 8 + 2 * j;
        const uint32_t b = e4m3x2(__fmul_rn(bf16_lo(w[j]), vi[d]), __fmul_rn(bf16_hi(w[j]), vi[d + 1]));
        reinterpret_cast<uint8_t*>(&vt[d][0])[tid] = (uint8_t)(b & 0xFF);
        reinterpret_cast<uint8_t*>(&vt[d + 1][0])[tid] = (uint8_t)(b >> 8);
      }
    }
    __syncthreads();
    uint4* dst = reinterpret_cast<uint4*>(vt8 + ((size_t)h * 128 + tid) * SP + (size_t)blk * 128);
#pragma unroll
    for (int k = 0; k < 8; ++k) dst[k] = make_uint4(vt[tid][4 * k], vt[tid][4 * k + 1], vt[tid][4 * k + 2], vt[tid][4 * k + 3]);
  }
}

// ------------------------------------------------------------------------------------------------ attention
struct AttnArgs {
  const float* qscale;   // [H][SP]
  const float* kscale;   // [H][SP/128]
  const float* vscale;   // [H][128]
  __nv_bfloat16* out;    // element (t, h, d) at out + t * ldo + h * 128 + d
  long long ldo;
  int S, SP, H;
};

constexpr int kAttnStages = 4;
// One 128-row query tile per CTA with two S buffers in TMEM, so QK^T of KV tile j + 1 runs on the tensor cores while
// the softmax of tile j does.  Warps 0-15: softmax, warp w on TMEM lane quadrant w % 4 and keys 32 (w / 4) .. +31 of
// each KV tile (four warps share each row: an FP8 tile leaves the softmax about half the MMA time a bf16 tile does);
// warp 16: TMA; warp 17: MMA.
constexpr int kAttnThreads = 576;
constexpr int kProdWarp = 16, kMmaWarp = 17;
constexpr int kQTile = 128;
constexpr float kTau = 2.0f;        // running-max lag allowed before O is rescaled (log2 units)
constexpr float kPOffset = 8.807354922057604f - kTau;   // log2(448) - tau
struct AttnSmem {
  static constexpr int TILE = 128 * 128;
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = TILE;                   // per stage: K, V^T
  static constexpr int KSC_OFF = KV_OFF + kAttnStages * 2 * TILE;   // this head's K-block scales
  static constexpr int MAX_KBLK = 2048;                                // sequences up to 262,144 tokens
  static constexpr int XCH_OFF = KSC_OFF + MAX_KBLK * 4;          // row-max exchange [2 parities][4 warps][128]
  static constexpr int LX_OFF = XCH_OFF + 2 * 4 * 128 * 4;         // row-sum exchange [4 warps][128]
  static constexpr int BAR_OFF = LX_OFF + 4 * 128 * 4;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}
// (exp2(a * scale - bias), exp2(b * scale - bias)) as f16x2 (a in the low half): one packed fp32 FMA, one packed
// conversion and one MUFU ex2 for two probabilities.  P is rounded to e4m3 next, so f16 precision is ample.
__device__ __forceinline__ uint32_t exp2_pair(float a, float b, uint64_t scale2, uint64_t nbias2) {
  uint32_t h;
  asm("{\n\t.reg .b64 x, y;\n\t.reg .f32 y0, y1;\n\t.reg .b32 hh;\n\t"
      "mov.b64 x, {%1, %2};\n\t"
      "fma.rn.f32x2 y, x, %3, %4;\n\t"
      "mov.b64 {y0, y1}, y;\n\t"
      "cvt.rn.f16x2.f32 hh, y1, y0;\n\t"
      "ex2.approx.f16x2 %0, hh;\n\t}"
      : "=r"(h)
      : "f"(a), "f"(b), "l"(scale2), "l"(nbias2));
  return h;
}
__device__ __forceinline__ uint64_t f32x2_splat(float v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float hsum2_f32(uint32_t h) {
  __half2 v = *reinterpret_cast<__half2*>(&h);
  return __low2float(v) + __high2float(v);
}
// two f16x2 pairs -> four e4m3 bytes (lo pair's low half in byte 0)
__device__ __forceinline__ uint32_t e4m3x4_f16(uint32_t lo, uint32_t hi) {
  uint16_t a, b;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(a) : "r"(lo));
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(b) : "r"(hi));
  return (uint32_t)a | ((uint32_t)b << 16);
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fp8_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
  using L = AttnSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + kAttnStages;
  uint64_t* kv_empty = v_full + kAttnStages;
  uint64_t* s_full = kv_empty + kAttnStages;   // [2]: QK^T of tile j in S buffer j % 2
  uint64_t* p_full = s_full + 2;               // [2]: P of tile j written over S buffer j % 2
  uint64_t* pv_done = p_full + 2;              // one phase per PV of a tile
  uint64_t* o_done = pv_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int q0 = blockIdx.x * kQTile;
  const int nkv = (p.S + 127) / 128;
  float* ksc_s = reinterpret_cast<float*>(smem + L::KSC_OFF);
  for (int i = threadIdx.x; i < nkv; i += blockDim.x) ksc_s[i] = p.kscale[(size_t)h * (p.SP / 128) + i];

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 16);   // one arrival per softmax warp
    }
    mbar_init(pv_done, 1);
    mbar_init(o_done, 1);
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S buffer 0 [0, 128), S buffer 1 [128, 256), O [256, 384).  P of keys 32k..32k+31 goes to columns
  // 32k..32k+7 of its S buffer (the columns the warp owning those keys read).

  if (warp == kProdWarp) {
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, L::TILE);
      tma_load_2d(smem + L::Q_OFF, &tmQ, 0, h * p.SP + q0, q_full);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % kAttnStages;
        const uint32_t ph = (j / kAttnStages) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, 201)) break;
        uint8_t* kv = smem + L::KV_OFF + st * 2 * L::TILE;
        mbar_arrive_expect_tx(&k_full[st], L::TILE);
        tma_load_2d(kv, &tmK, 0, h * p.SP + j * 128, &k_full[st]);
        mbar_arrive_expect_tx(&v_full[st], L::TILE);
        tma_load_2d(kv + L::TILE, &tmV, j * 128, h * 128, &v_full[st]);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_fp8(128, 128);
      const uint32_t qs = smem_u32(smem + L::Q_OFF);
      auto issue_s = [&](int b, int st) {
        const uint32_t ks = smem_u32(smem + L::KV_OFF + st * 2 * L::TILE);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          mma_fp8_ss(tmem + b * 128, sdesc_kmajor_sw128(qs + kb * 32), sdesc_kmajor_sw128(ks + kb * 32), idesc, kb != 0);
      };
      auto issue_pv = [&](int b, int st, int j) {
        const uint32_t vs = smem_u32(smem + L::KV_OFF + st * 2 * L::TILE + L::TILE);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          mma_fp8_ts(tmem + 256, tmem + b * 128 + kb * 32, sdesc_kmajor_sw128(vs + kb * 32), idesc, (j | kb) != 0);
      };
      bool ok = mbar_wait(q_full, 0, 202);
      for (int j = 0; ok && j < 2 && j < nkv; ++j) {   // prologue: S of tiles 0 and 1
        if (!(ok = mbar_wait(&k_full[j], 0, 203))) break;
        tc_fence_after();
        issue_s(j, j);
        tc_commit(&s_full[j]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int b = j & 1, st = j % kAttnStages;
        if (!(ok = mbar_wait(&p_full[b], (j >> 1) & 1, 204) && mbar_wait(&v_full[st], (j / kAttnStages) & 1, 205)))
          break;
        tc_fence_after();
        issue_pv(b, st, j);
        tc_commit(pv_done);
        tc_commit(&kv_empty[st]);
        if (j + 2 < nkv) {
          const int st2 = (j + 2) % kAttnStages;
          if (!(ok = mbar_wait(&k_full[st2], ((j + 2) / kAttnStages) & 1, 206))) break;
          tc_fence_after();
          issue_s(b, st2);   // after PV(j) in issue order, so P(j) is consumed before S(j + 2) overwrites it
          tc_commit(&s_full[b]);
        }
      }
      tc_commit(o_done);
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int kq = warp >> 2;        // keys 32 kq .. 32 kq + 31 of each tile, O columns 32 kq .. 32 kq + 31
    const int qd = warp & 3;         // TMEM lane quadrant
    const int r = qd * 32 + lane;
    const int query = q0 + r;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t o_col = tmem + lane_off + 256 + kq * 32;
    const int bar_id = 1 + qd;       // named barrier of the four warps sharing these rows
    float* xch = reinterpret_cast<float*>(smem + L::XCH_OFF);
    float* lx = reinterpret_cast<float*>(smem + L::LX_OFF);
    const float qr = p.qscale[(size_t)h * p.SP + query];
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int b = j & 1;
      const uint32_t s_col = tmem + lane_off + b * 128 + kq * 32;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (j >> 1) & 1, 210));
      const float scale = qr * ksc_s[j];
      const int valid = p.S - j * 128 - kq * 32;   // keys of this warp's slice inside the sequence
      uint32_t sr[32];
      float mloc = -INFINITY;
      if (ok) {
        tc_fence_after();
        tmem_ld32(s_col, sr);
        tmem_ld_wait();
        if (valid < 32) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e >= valid) sr[e] = __float_as_uint(-INFINITY);
        }
        float m[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t* f = sr + 8 * k;
          m[k] = max3(max3(__uint_as_float(f[0]), __uint_as_float(f[1]), __uint_as_float(f[2])),
                      max3(__uint_as_float(f[3]), __uint_as_float(f[4]), __uint_as_float(f[5])),
                      fmaxf(__uint_as_float(f[6]), __uint_as_float(f[7])));
        }
        mloc = fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
      }
      float* xs = xch + (j & 1) * 512;
      xs[kq * 128 + r] = mloc;
      // exchange the four partial maxima; the barrier also ANDs the warps' wait results, so the four warps sharing
      // these rows leave the loop together (a named barrier has no timeout)
      {
        uint32_t all;
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred p, %2, 128, p;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(all)
            : "r"((uint32_t)ok), "r"(bar_id)
            : "memory");
        ok = all != 0;
      }
      if (!ok) break;
      const float mx = fmaxf(fmaxf(xs[r], xs[128 + r]), fmaxf(xs[256 + r], xs[384 + r]));
      const float mnew = mx * scale;
      // raise the running max only when a row's max grew by more than tau; the tcgen05 ld/st of O are warp-wide,
      // so a warp rescales when any of its rows must (the others multiply by 1); each warp rescales its 32 columns
      // once the previous tile's PV has landed
      const bool need = mnew > m_used + kTau;
      float alpha = 1.0f;
      if (need && j > 0) alpha = ex2(m_used - mnew);
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // a wait that gives up has recorded the error; the warp stays in step with its partners
        __all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, 213));
        tc_fence_after();
        uint32_t o[32];
        tmem_ld32(o_col, o);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
        tmem_st32(o_col, o);
      }
      if (need) {
        l *= alpha;
        m_used = mnew;
      }
      const uint64_t scale2 = f32x2_splat(scale), nbias2 = f32x2_splat(kPOffset - m_used);
      uint32_t pw[8];
      uint32_t hs0 = 0, hs1 = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const uint32_t e0 = exp2_pair(__uint_as_float(sr[4 * w]), __uint_as_float(sr[4 * w + 1]), scale2, nbias2);
        const uint32_t e1 = exp2_pair(__uint_as_float(sr[4 * w + 2]), __uint_as_float(sr[4 * w + 3]), scale2, nbias2);
        hs0 = hadd2(hs0, e0);
        hs1 = hadd2(hs1, e1);
        pw[w] = e4m3x4_f16(e0, e1);
      }
      tmem_st8(s_col, pw);
      l += hsum2_f32(hadd2(hs0, hs1));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    // ---- epilogue: row sum over the four warps, then this warp's 32 columns of O / l * vscale -> bf16
    lx[kq * 128 + r] = l;
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
    const float lt = (lx[r] + lx[128 + r]) + (lx[256 + r] + lx[384 + r]);
    ok = ok && mbar_wait(o_done, 0, 212);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      const float inv_l = 1.0f / lt;
      const float* vs = p.vscale + h * 128 + kq * 32;
      uint32_t o[32];
      tmem_ld32(o_col, o);
      tmem_ld_wait();
      if (query < p.S) {
        uint4* d4 = reinterpret_cast<uint4*>(p.out + (long long)query * p.ldo + h * 128 + kq * 32);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o[q4 * 8 + e]) * inv_l * vs[q4 * 8 + e];
          d4[q4] = make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]),
                              pack_bf16(f[6], f[7]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 512);
}

}  // namespace h3
