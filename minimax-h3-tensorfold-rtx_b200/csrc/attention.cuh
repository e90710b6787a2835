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

__global__ void __launch_bounds__(256) qknorm_rope_kernel(QkNormArgs a) {
  const int lane = threadIdx.x & 31;
  const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long nrows = (long long)a.S * 2 * a.H;
  if (wid >= nrows) return;
  const int s = (int)(wid / (2 * a.H));
  const int rem = (int)(wid % (2 * a.H));
  const int which = rem / a.H, h = rem % a.H;
  __nv_bfloat16* row = (which ? a.k : a.q) + (long long)s * a.ld + h * 128;
  const float* w = which ? a.kw : a.qw;
  uint2 u = *reinterpret_cast<const uint2*>(row + lane * 4);
  float x[4] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y)};
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
#pragma unroll
  for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), a.eps)));
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) y[e] = __fmul_rn(__fmul_rn(x[e], r), w[lane * 4 + e]);
  const int half = a.rot >> 1, hq = half >> 2;
  const int d0 = lane * 4;
  int src = lane;
  if (d0 < half) src = lane + hq;
  else if (d0 < a.rot) src = lane - hq;
  float pv[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) pv[e] = __shfl_sync(0xffffffffu, y[e], src);
  float o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = d0 + e;
    if (d < half) {
      float4 f = *reinterpret_cast<const float4*>(a.rope + ((size_t)s * half + d) * 4);
      o[e] = __fadd_rn(__fmul_rn(f.x, y[e]), __fmul_rn(f.y, pv[e]));
    } else if (d < a.rot) {
      float4 f = *reinterpret_cast<const float4*>(a.rope + ((size_t)s * half + (d - half)) * 4);
      o[e] = __fadd_rn(__fmul_rn(f.z, pv[e]), __fmul_rn(f.w, y[e]));
    } else {
      o[e] = y[e];
    }
  }
  *reinterpret_cast<uint2*>(row + lane * 4) = make_uint2(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]));
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
  const int blk = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int t0 = blk * 128, t1 = min(S, t0 + 128);
  float ks = 0.f, vm = 0.f;
  for (int t = t0; t < t1; ++t) {
    const long long off = (long long)t * a.ld + (long long)h * a.hstride + d;
    ks = __fadd_rn(ks, __bfloat162float(a.k[off]));
    vm = fmaxf(vm, fabsf(__bfloat162float(a.v[off])));
  }
  ksum_part[((size_t)blk * H + h) * 128 + d] = ks;
  vmax_part[((size_t)blk * H + h) * 128 + d] = vm;
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
  // ---- V (per channel), transposed
  {
    const float* vi = vinv + h * 128;
    uint8_t* dst = vt8 + (size_t)h * 128 * SP + t;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 u = live ? *reinterpret_cast<const uint4*>(a.v + base + c * 8) : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = c * 8 + 2 * j;
        uint32_t b = e4m3x2(__fmul_rn(bf16_lo(w[j]), vi[d]), __fmul_rn(bf16_hi(w[j]), vi[d + 1]));
        dst[(size_t)d * SP] = (uint8_t)(b & 0xFF);
        dst[(size_t)(d + 1) * SP] = (uint8_t)(b >> 8);
      }
    }
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

constexpr int kAttnStages = 3;
// warps 0-15: softmax, warp w on query tile w / 8, keys 64 * (w / 4 % 2) .. +63 of each KV tile, TMEM lane quadrant
// w % 4; warp 16: TMA; warp 17: MMA.  Two warps share each row (one per half of the keys): an FP8 tile gives the
// softmax only about half the MMA time a bf16 tile does, so each row's work is split.
constexpr int kAttnThreads = 576;
constexpr int kProdWarp = 16, kMmaWarp = 17;
constexpr float kTau = 2.0f;        // running-max lag allowed before O is rescaled (log2 units)
constexpr float kPOffset = 8.807354922057604f - kTau;   // log2(448) - tau
struct AttnSmem {
  static constexpr int TILE = 128 * 128;
  static constexpr int Q_OFF = 0;                       // Q0, Q1
  static constexpr int KV_OFF = 2 * TILE;               // per stage: K, V^T
  static constexpr int KSC_OFF = KV_OFF + kAttnStages * 2 * TILE;   // this head's K-block scales
  static constexpr int MAX_KBLK = 2048;                                // sequences up to 262,144 tokens
  static constexpr int XCH_OFF = KSC_OFF + MAX_KBLK * 4;          // row-max exchange [2 parities][2 tiles][2][128]
  static constexpr int LX_OFF = XCH_OFF + 2 * 2 * 2 * 128 * 4;     // row-sum exchange [2 tiles][2][128]
  static constexpr int BAR_OFF = LX_OFF + 2 * 2 * 128 * 4;
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
  uint64_t* s_full = kv_empty + kAttnStages;   // [2]
  uint64_t* p_full = s_full + 2;               // [2]
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int q0 = blockIdx.x * 256;
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
    }
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
  // TMEM columns: S0 [0, 128), S1 [128, 256), O0 [256, 384), O1 [384, 512); P_i overwrites S_i's first 32 columns.

  if (warp == kProdWarp) {
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, 2 * L::TILE);
      tma_load_2d(smem + L::Q_OFF, &tmQ, 0, h * p.SP + q0, q_full);
      tma_load_2d(smem + L::Q_OFF + L::TILE, &tmQ, 0, h * p.SP + q0 + 128, q_full);
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
      const uint32_t qs0 = smem_u32(smem + L::Q_OFF), qs1 = qs0 + L::TILE;
      auto issue_s = [&](int i, int st) {
        const uint32_t ks = smem_u32(smem + L::KV_OFF + st * 2 * L::TILE);
        const uint32_t qs = i ? qs1 : qs0;
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          mma_fp8_ss(tmem + i * 128, sdesc_kmajor_sw128(qs + kb * 32), sdesc_kmajor_sw128(ks + kb * 32), idesc, kb != 0);
      };
      // P of keys 32 kb .. 32 kb + 31 sits in TMEM columns 64 (kb / 2) + 8 (kb % 2) of S_i (each half of the
      // keys writes its P into its own S columns)
      auto issue_pv = [&](int i, int st, int j) {
        const uint32_t vs = smem_u32(smem + L::KV_OFF + st * 2 * L::TILE + L::TILE);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          mma_fp8_ts(tmem + 256 + i * 128, tmem + i * 128 + (kb >> 1) * 64 + (kb & 1) * 8,
                     sdesc_kmajor_sw128(vs + kb * 32), idesc, (j | kb) != 0);
      };
      bool ok = mbar_wait(q_full, 0, 202) && mbar_wait(&k_full[0], 0, 203);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        tc_commit(&s_full[0]);
        issue_s(1, 0);
        tc_commit(&s_full[1]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j % kAttnStages;
        const uint32_t ph = (j / kAttnStages) & 1;
        if (!(ok = mbar_wait(&p_full[0], j & 1, 204) && mbar_wait(&v_full[st], ph, 205))) break;
        tc_fence_after();
        issue_pv(0, st, j);
        const bool more = j + 1 < nkv;
        const int st1 = (j + 1) % kAttnStages;
        if (more) {
          if (!(ok = mbar_wait(&k_full[st1], ((j + 1) / kAttnStages) & 1, 206))) break;
          tc_fence_after();
          issue_s(0, st1);
          tc_commit(&s_full[0]);
        }
        if (!(ok = mbar_wait(&p_full[1], j & 1, 207))) break;
        tc_fence_after();
        issue_pv(1, st, j);
        tc_commit(&kv_empty[st]);
        if (more) {
          issue_s(1, st1);
          tc_commit(&s_full[1]);
        }
      }
      tc_commit(o_done);
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int i = warp >> 3;          // query tile
    const int hf = (warp >> 2) & 1;   // which 64 keys of each KV tile (and which 64 columns of O)
    const int qd = warp & 3;          // TMEM lane quadrant
    const int r = qd * 32 + lane;
    const int query = q0 + i * 128 + r;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t s_col = tmem + lane_off + i * 128;
    const uint32_t o_col = tmem + lane_off + 256 + i * 128 + hf * 64;
    const int bar_id = 1 + i * 4 + qd;   // named barrier of the warp pair (w, w ^ 4) sharing these rows
    float* xch = reinterpret_cast<float*>(smem + L::XCH_OFF);
    float* lx = reinterpret_cast<float*>(smem + L::LX_OFF);
    const float qr = p.qscale[(size_t)h * p.SP + query];
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      ok = mbar_wait(&s_full[i], j & 1, 210 + i);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const float scale = qr * ksc_s[j];
      const int valid = p.S - j * 128 - hf * 64;   // keys of this half inside the sequence
      // pass 1: this half's row max (keys past S masked in the last tile), then the pair's max through smem
      float mh = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sr[32];
        tmem_ld32(s_col + hf * 64 + c * 32, sr);
        tmem_ld_wait();
        if (valid < 64) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= valid) sr[e] = __float_as_uint(-INFINITY);
        }
        float m[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t* f = sr + 8 * k;
          m[k] = max3(max3(__uint_as_float(f[0]), __uint_as_float(f[1]), __uint_as_float(f[2])),
                      max3(__uint_as_float(f[3]), __uint_as_float(f[4]), __uint_as_float(f[5])),
                      fmaxf(__uint_as_float(f[6]), __uint_as_float(f[7])));
        }
        mh = max3(mh, fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
      }
      float* xs = xch + ((j & 1) * 2 + i) * 256;
      xs[hf * 128 + r] = mh;
      asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
      const float mx = fmaxf(mh, xs[(hf ^ 1) * 128 + r]);
      const float mnew = mx * scale;
      // raise the running max only when a row's max grew by more than tau; the tcgen05 ld/st of O are warp-wide,
      // so a warp rescales when any of its rows must (the others multiply by 1); each half rescales its 64 columns
      const bool need = mnew > m_used + kTau;
      float alpha = 1.0f;
      if (need && j > 0) alpha = ex2(m_used - mnew);
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(o_col + c * 32, o);
        }
        tmem_st_wait();
      }
      if (need) {
        l *= alpha;
        m_used = mnew;
      }
      const uint64_t scale2 = f32x2_splat(scale), nbias2 = f32x2_splat(kPOffset - m_used);
      // pass 2: P = exp2(s * scale - m + c) -> e4m3 into this half's own S columns 64 hf .. 64 hf + 15 (chunk c's P
      // words overwrite columns of chunk 0, which was read first)
      uint32_t hs0 = 0, hs1 = 0;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sr[32];
        tmem_ld32(s_col + hf * 64 + c * 32, sr);
        tmem_ld_wait();
        if (valid < 64) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= valid) sr[e] = __float_as_uint(-INFINITY);
        }
        uint32_t pw[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const uint32_t e0 = exp2_pair(__uint_as_float(sr[4 * w]), __uint_as_float(sr[4 * w + 1]), scale2, nbias2);
          const uint32_t e1 = exp2_pair(__uint_as_float(sr[4 * w + 2]), __uint_as_float(sr[4 * w + 3]), scale2, nbias2);
          hs0 = hadd2(hs0, e0);
          hs1 = hadd2(hs1, e1);
          pw[w] = e4m3x4_f16(e0, e1);
        }
        tmem_st8(s_col + hf * 64 + c * 8, pw);
      }
      l += hsum2_f32(hadd2(hs0, hs1));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[i]);
    }
    // ---- epilogue: row sum of both halves, then this half's 64 columns of O / l * vscale -> bf16
    lx[(i * 2 + hf) * 128 + r] = l;
    asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
    const float lt = l + lx[(i * 2 + (hf ^ 1)) * 128 + r];
    ok = ok && mbar_wait(o_done, 0, 212);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      const float inv_l = 1.0f / lt;
      const float* vs = p.vscale + h * 128 + hf * 64;
      __nv_bfloat16* dst = p.out + (long long)query * p.ldo + h * 128 + hf * 64;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        __syncwarp();
        tmem_ld32(o_col + c * 32, o);
        tmem_ld_wait();
        if (query < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o[q4 * 8 + e]) * inv_l * vs[c * 32 + q4 * 8 + e];
            d4[q4] = make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]),
                                pack_bf16(f[6], f[7]));
          }
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
