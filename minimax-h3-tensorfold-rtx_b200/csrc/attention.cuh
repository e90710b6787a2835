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
// Per (token, q|k, head) row of Dh = 128, lane l of the token's warp owns dims 4l..4l+3.
// y = x / sqrt(mean(x^2) + eps) * w; pair i < rot/2 couples dims i and i + rot/2 through the token's 2x2 matrix
// rope[s, i] (o_i = f00 y_i + f01 y_j, o_j = f10 y_i + f11 y_j); dims >= rot pass through.  In place on the bf16 rows.
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
// rows.  Rows go in groups of eight (q and k of four heads), all eight loaded before any is written back: the rows
// live in one buffer, so a load placed after a store could not be moved ahead of it, and one row in flight at a time
// leaves the HBM pipe mostly idle.
//
// Per group the sums of squares are reduced over the warp transposed: at each xor stage a lane sends the half of its
// rows it gives up and adds the partner's half of the rows it keeps, so the five stages cost 9 shuffles for eight rows
// instead of 40, and each lane ends with one row's sum (the same pairwise tree as a per-row xor butterfly, so the same
// bits).  Each lane then takes one IEEE sqrt and division for that row and the eight 1/rms values are broadcast back.
// The rotation is branch-free: a lane's four dims are all in the first half, all in the second, or all past `rot`, so
// o = ca * y + cb * y_partner with per-lane coefficients (fp addition commutes, so f10 * y_i + f11 * y_j is the same
// value in either order), and dims past `rot` keep y.
__device__ __forceinline__ float sumsq4(uint2 u) {
  const float x[4] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y)};
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
  return ss;
}

// p[j]: this lane's partial sum of row j -> the warp sum of row (4 (lane>>4 & 1) + 2 (lane>>3 & 1) + (lane>>2 & 1)).
__device__ __forceinline__ float warp_sum8_transposed(const float (&p)[8], int lane) {
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
  float q[4], r[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float keep = b16 ? p[4 + i] : p[i], send = b16 ? p[i] : p[4 + i];
    q[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float keep = b8 ? q[2 + i] : q[i], send = b8 ? q[i] : q[2 + i];
    r[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
  float s;
  {
    const float keep = b4 ? r[1] : r[0], send = b4 ? r[0] : r[1];
    s = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
  return s;
}

// p[j]: this lane's partial max of row j -> the warp max of row (4 (lane>>4 & 1) + 2 (lane>>3 & 1) + (lane>>2 & 1)),
// by the same transposed exchange (max is exact, so any order gives the same value)
__device__ __forceinline__ float warp_max8_transposed(const float (&p)[8], int lane) {
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
  float q[4], r[2];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    q[i] = fmaxf(b16 ? p[4 + i] : p[i], __shfl_xor_sync(0xffffffffu, b16 ? p[i] : p[4 + i], 16));
#pragma unroll
  for (int i = 0; i < 2; ++i)
    r[i] = fmaxf(b8 ? q[2 + i] : q[i], __shfl_xor_sync(0xffffffffu, b8 ? q[i] : q[2 + i], 8));
  float s = fmaxf(b4 ? r[1] : r[0], __shfl_xor_sync(0xffffffffu, b4 ? r[0] : r[1], 4));
  s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, 2));
  return fmaxf(s, __shfl_xor_sync(0xffffffffu, s, 1));
}

__device__ __forceinline__ uint2 qk_row(uint2 u, const float* w, const float (&ca)[4], const float (&cb)[4],
                                        bool rotated, int src, float r) {
  const float x[4] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y)};
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) y[e] = __fmul_rn(__fmul_rn(x[e], r), w[e]);
  float o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float pv = __shfl_sync(0xffffffffu, y[e], src);
    const float t = __fadd_rn(__fmul_rn(ca[e], y[e]), __fmul_rn(cb[e], pv));
    o[e] = rotated ? t : y[e];
  }
  return make_uint2(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]));
}

__global__ void __launch_bounds__(256) qknorm_rope_kernel(QkNormArgs a) {
  const int lane = threadIdx.x & 31;
  const int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (s >= a.S) return;
  const int half = a.rot >> 1, hq = half >> 2;
  const int d0 = lane * 4;
  const bool first = d0 < half, rotated = d0 < a.rot;
  const int src = first ? lane + hq : (rotated ? lane - hq : lane);
  // o_i = f00 y_i + f01 y_j (first half), o_j = f11 y_j + f10 y_i (second half) for pair (i, j = i + rot/2)
  float ca[4], cb[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = d0 + e;
    const int pair = first ? d : d - half;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rotated) v = *reinterpret_cast<const float4*>(a.rope + ((size_t)s * half + pair) * 4);
    ca[e] = first ? v.x : v.w;
    cb[e] = first ? v.y : v.z;
  }
  float qw[4], kw[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    qw[e] = a.qw[d0 + e];
    kw[e] = a.kw[d0 + e];
  }
  __nv_bfloat16* qrow = a.q + (long long)s * a.ld + d0;
  __nv_bfloat16* krow = a.k + (long long)s * a.ld + d0;
  for (int h0 = 0; h0 < a.H; h0 += 4) {
    uint2 u[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      u[2 * j] = u[2 * j + 1] = make_uint2(0u, 0u);
      if (h0 + j < a.H) {
        u[2 * j] = *reinterpret_cast<const uint2*>(qrow + (h0 + j) * 128);
        u[2 * j + 1] = *reinterpret_cast<const uint2*>(krow + (h0 + j) * 128);
      }
    }
    float p[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = sumsq4(u[j]);
    const float ss = warp_sum8_transposed(p, lane);
    const float rmine = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), a.eps)));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (h0 + j < a.H) {
        const int kq = 2 * j, kk = 2 * j + 1;   // row k is held by lane 16 (k>>2) + 8 (k>>1 & 1) + 4 (k & 1)
        const float rq = __shfl_sync(0xffffffffu, rmine, ((kq >> 2) << 4) | (((kq >> 1) & 1) << 3) | ((kq & 1) << 2));
        const float rk = __shfl_sync(0xffffffffu, rmine, ((kk >> 2) << 4) | (((kk >> 1) & 1) << 3) | ((kk & 1) << 2));
        *reinterpret_cast<uint2*>(qrow + (h0 + j) * 128) = qk_row(u[kq], qw, ca, cb, rotated, src, rq);
        *reinterpret_cast<uint2*>(krow + (h0 + j) * 128) = qk_row(u[kk], kw, ca, cb, rotated, src, rk);
      }
    }
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
  // eight blocks' partials are loaded before any is added (one load in flight at a time made this a chain of
  // memory latencies, 43 us at S = 37,760); the sum keeps its block order
  for (int b0 = 0; b0 < nblk; b0 += 8) {
    float kp[8], vp[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool in = b0 + j < nblk;
      kp[j] = in ? ksum_part[(size_t)(b0 + j) * H * 128 + i] : 0.f;
      vp[j] = in ? vmax_part[(size_t)(b0 + j) * H * 128 + i] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (b0 + j < nblk) {
        ks = __fadd_rn(ks, kp[j]);
        vm = fmaxf(vm, vp[j]);
      }
    }
  }
  kmean[i] = __fdiv_rn(ks, (float)S);
  vm = fmaxf(vm, 1e-30f);
  vscale[i] = __fdiv_rn(vm, 448.0f);
  vinv[i] = __fdiv_rn(448.0f, vm);
}

// Per (128-token block, head): Q row -> e4m3 [H][SP][128] + fp32 scale [H][SP]; K row (smoothed) -> e4m3 with one
// scale per block [H][SP/128]; V -> e4m3 transposed [H][128][SP] (keys contiguous, the K-major B operand of PV).  Rows
// t >= S are written as zeros.  Warp w takes rows 32 w .. 32 w + 31, one row at a time across its lanes (lane l owns
// dims 4 l .. 4 l + 3), so every load is one 256-byte row and every e4m3 store one 128-byte row.  K is read twice (its
// block max first; the second read comes from L2).  V goes through a shared-memory tile [d][t] four tokens at a time,
// then leaves as 128-byte rows of the transpose.
__global__ void __launch_bounds__(128) attn_quant_kernel(AttnView a, int S, int SP, int H, const float* kmean,
                                                         const float* vinv, uint8_t* q8, float* qscale, uint8_t* k8,
                                                         float* kscale, uint8_t* vt8) {
  __shared__ float red[4];
  __shared__ uint32_t vt[128][33];   // [d][t / 4] words of e4m3 V (byte t % 4), padded
  const int blk = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int d0 = lane * 4;
  const float qmul = kLog2e / sqrtf(128.0f);
  auto row_ptr = [&](const __nv_bfloat16* base, int t) {
    return reinterpret_cast<const uint2*>(base + (long long)t * a.ld + (long long)h * a.hstride + d0);
  };
  auto load4 = [&](const __nv_bfloat16* base, int t, float (&x)[4]) {
    const uint2 u = t < S ? *row_ptr(base, t) : make_uint2(0, 0);
    x[0] = bf16_lo(u.x);
    x[1] = bf16_hi(u.x);
    x[2] = bf16_lo(u.y);
    x[3] = bf16_hi(u.y);
  };
  auto pack4 = [](const float (&y)[4], float inv) {
    return e4m3x2(__fmul_rn(y[0], inv), __fmul_rn(y[1], inv)) |
           (e4m3x2(__fmul_rn(y[2], inv), __fmul_rn(y[3], inv)) << 16);
  };
  // ---- Q: one fp32 scale per row, eight rows at a time: the row maxima are reduced transposed (each lane ends with
  // one row's max), so each lane makes the scale's two IEEE divisions for one row instead of all lanes for every row
#pragma unroll 1
  for (int i0 = 0; i0 < 32; i0 += 8) {
    const int t0 = blk * 128 + warp * 32 + i0;
    float x[8][4], pm[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      load4(a.q, t0 + r, x[r]);
      pm[r] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[r][j] = __fmul_rn(x[r][j], qmul);
        pm[r] = fmaxf(pm[r], fabsf(x[r][j]));
      }
    }
    const int mine = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);   // the row this lane ends with
    const float qr_mine = __fdiv_rn(fmaxf(warp_max8_transposed(pm, lane), 1e-30f), 448.0f);
    const float qi_mine = __fdiv_rn(1.0f, qr_mine);
    if ((lane & 3) == 0) qscale[(size_t)h * SP + t0 + mine] = qr_mine;   // tiny but finite for padded rows
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int src = ((r >> 2) << 4) | (((r >> 1) & 1) << 3) | ((r & 1) << 2);
      const float qi = __shfl_sync(0xffffffffu, qi_mine, src);
      reinterpret_cast<uint32_t*>(q8 + ((size_t)h * SP + t0 + r) * 128)[lane] = pack4(x[r], qi);
    }
  }
  // ---- K (smoothed by the sequence mean, one scale per 128-key block)
  float km[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) km[j] = kmean[h * 128 + d0 + j];
  auto smooth = [&](int t, float (&x)[4]) {
    load4(a.k, t, x);
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = t < S ? __fsub_rn(x[j], km[j]) : 0.f;
  };
  float kmax = 0.f;
#pragma unroll 4
  for (int i = 0; i < 32; ++i) {
    float x[4];
    smooth(blk * 128 + warp * 32 + i, x);
#pragma unroll
    for (int j = 0; j < 4; ++j) kmax = fmaxf(kmax, fabsf(x[j]));
  }
  kmax = warp_max(kmax);
  if (lane == 0) red[warp] = kmax;
  __syncthreads();
  kmax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float kr = __fdiv_rn(fmaxf(kmax, 1e-30f), 448.0f);
  const float kinv = __fdiv_rn(1.0f, kr);
#pragma unroll 4
  for (int i = 0; i < 32; ++i) {
    const int t = blk * 128 + warp * 32 + i;
    float x[4];
    smooth(t, x);
    reinterpret_cast<uint32_t*>(k8 + ((size_t)h * SP + t) * 128)[lane] = pack4(x, kinv);
  }
  if (tid == 0) kscale[(size_t)h * (SP / 128) + blk] = kr;
  // ---- V (per channel), transposed: four tokens at a time into the [d][t] tile, then 128-byte rows out
  float vi[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) vi[j] = vinv[h * 128 + d0 + j];
#pragma unroll 2
  for (int i = 0; i < 32; i += 4) {
    uint32_t bytes[4] = {0u, 0u, 0u, 0u};   // dim d0 + j of tokens i .. i + 3, byte k for token i + k
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float x[4];
      load4(a.v, blk * 128 + warp * 32 + i + k, x);
      const uint32_t lo = e4m3x2(__fmul_rn(x[0], vi[0]), __fmul_rn(x[1], vi[1]));
      const uint32_t hi = e4m3x2(__fmul_rn(x[2], vi[2]), __fmul_rn(x[3], vi[3]));
      bytes[0] |= (lo & 0xFFu) << (8 * k);
      bytes[1] |= (lo >> 8) << (8 * k);
      bytes[2] |= (hi & 0xFFu) << (8 * k);
      bytes[3] |= (hi >> 8) << (8 * k);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) vt[d0 + j][(warp * 32 + i) / 4] = bytes[j];
  }
  __syncthreads();
#pragma unroll 4
  for (int r = 0; r < 32; ++r) {
    const int d = warp * 32 + r;
    reinterpret_cast<uint32_t*>(vt8 + ((size_t)h * 128 + d) * SP + (size_t)blk * 128)[lane] = vt[d][lane];
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
  // Block-sparse mask (NULL = dense): the KV tiles query tile qt attends to are kv_idx[kv_ptr[qt] .. kv_ptr[qt+1]),
  // 128-token tiles, shared by all heads.  Sparse launches take one query tile per CTA (NT = 1).
  const int* kv_ptr;
  const int* kv_idx;
  // Output to peers (ranks > 0, Ulysses): token t's row goes to peer[t / n_local] at row rank * n_local + t % n_local
  // (row length ldo) instead of to out.
  unsigned long long peer[8];
  int ranks, rank, n_local;
};

// One CTA = NT 128-row query tiles (A, B) of one head: NT = 2 for dense launches; NT = 1 for block-sparse ones,
// whose query tiles each walk their own KV list, and which then run two CTAs per SM, so that every SM sub-partition
// still holds two softmax warps.  Each 128-key KV tile is taken in two 64-key halves, and each query tile has two
// 64-column S buffers in TMEM (one per half), so QK^T of the next half runs on the tensor cores while the softmax of
// this one does: a group of MMAs takes several hundred cycles from issue to its commit, which then never sits in
// series with the softmax.  Warps 0-3: softmax of tile A, warps 4-7: tile B -- warp w on TMEM lane quadrant w % 4,
// one thread per query row, so the row max needs no exchange between threads; warp 4 NT: TMA; warps 4 NT + 1 + t:
// MMA of tile t (an issuing thread that stops at a barrier lets the tensor pipe run dry; two keep it fed).
// TMEM columns (NT = 2): S_A [0, 64) and [64, 128), S_B [128, 192) and [192, 256), O_A [256, 384), O_B [384, 512);
// (NT = 1): S_A [0, 128), O_A [128, 256).  P of keys 32c..32c+31 of a half (e4m3) is written over columns
// 32c..32c+7 of its S buffer.
constexpr int kQTile = 128;
__host__ __device__ constexpr int attn_stages(int nt) { return nt == 2 ? 4 : 2; }    // K/V smem ring depth
__host__ __device__ constexpr int attn_threads(int nt) { return 160 * nt + 32; }   // 5 warps a tile + TMA warp
// Running-max lag allowed before O is rescaled (log2 units).  P of a row then stays within [2^-tau, 1] x 448 of
// its max half by half, and O and l are rescaled only when a max grows by more than 2^tau.  6 against 2: block-sparse
// 5.79 -> 5.47 ms at S = 37,760, H = 40 (its KV lists raise row maxima more often), dense unchanged; cosine against
// fp32 SDPA unchanged to 1e-5 (0.99867 dense, 0.99863 sparse at S = 4096, H = 4).
constexpr float kTau = 6.0f;
constexpr float kPOffset = 8.807354922057604f - kTau;   // log2(448) - tau
// Pairs of each 32-key chunk whose exp2 runs as a polynomial on the FMA pipe instead of the MUFU (bit i: keys 2i,
// 2i + 1).  The MUFU completes 16 ex2 per cycle per SM, which alone would bound an FP8 tile's softmax at twice the
// tile's MMA time; moving part of the exponentials to the FMA pipe shortens it.  Five of the 16 pairs, every third
// one, measured best at S = 37,760, H = 40: 21.14 ms, against 21.36-21.47 for six spaced by three and 21.71 for six
// in pairs of neighbours (0x5252), in one run.
constexpr uint32_t kPolyPairs = 0x2492u;
template <int NT>
struct AttnSmem {
  static constexpr int TILE = 128 * 128;
  static constexpr int Q_OFF = 0;                                      // Q tiles A, B
  static constexpr int KV_OFF = NT * TILE;                              // per stage: K, V^T
  static constexpr int KSC_OFF = KV_OFF + attn_stages(NT) * 2 * TILE;   // this head's K-block scales
  static constexpr int MAX_KBLK = 2048;                                 // sequences up to 262,144 tokens
  static constexpr int KVT_OFF = KSC_OFF + MAX_KBLK * 4;                // KV tile of each step (block-sparse)
  static constexpr int BAR_OFF = KVT_OFF + MAX_KBLK * 4;
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
__device__ __forceinline__ uint64_t f32x2_splat(float v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(v));
  return r;
}
__device__ __forceinline__ uint64_t f32x2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f32x2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// 2^x for a pair, by range reduction x = n + g (n = round(x), |g| <= 1/2) and a degree-3 polynomial for 2^g (a
// relative-error least-squares fit on [-1/2, 1/2]; max relative error 7.5e-5, below the e4m3 rounding P gets next
// by three orders of magnitude).  n comes from the magic-number rounding x + (1.5 * 2^23 + 127): the sum's low
// mantissa bits hold 127 + n, which shifted into the exponent field is the fp32 2^n.  x is clamped to >= -126.
__device__ __forceinline__ uint64_t exp2_poly_pair(uint64_t x2) {
  constexpr float kMagic = 12582912.0f + 127.0f;
  float a, b;
  f32x2_unpack(x2, a, b);
  const uint64_t x = f32x2_pack(fmaxf(a, -126.0f), fmaxf(b, -126.0f));
  const uint64_t t = add2(x, f32x2_splat(kMagic));
  const uint64_t n = add2(t, f32x2_splat(-kMagic));
  const uint64_t g = fma2(n, f32x2_splat(-1.0f), x);
  uint64_t p = fma2(f32x2_splat(0.0551716685295105f), g, f32x2_splat(0.2426111400127411f));
  p = fma2(p, g, f32x2_splat(0.6932609677314758f));
  p = fma2(p, g, f32x2_splat(0.9999280571937561f));
  float t0, t1;
  f32x2_unpack(t, t0, t1);
  return mul2(p, f32x2_pack(__uint_as_float(__float_as_uint(t0) << 23), __uint_as_float(__float_as_uint(t1) << 23)));
}
__device__ __forceinline__ uint64_t exp2_mufu_pair(uint64_t x2) {
  float a, b;
  f32x2_unpack(x2, a, b);
  return f32x2_pack(ex2(a), ex2(b));
}
// 32 scores of one row -> 8 words of e4m3 P = exp2(s * scale - bias) (key 4w + i in byte i of word w); l2 += the
// unrounded P (two fp32 lanes).
__device__ __forceinline__ void p_chunk(const uint32_t (&s)[32], uint64_t scale2, uint64_t nbias2, uint32_t (&pw)[8],
                                        uint64_t& l2a, uint64_t& l2b) {
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    uint64_t y[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int pi = 2 * w + hh;
      const uint64_t x = fma2(f32x2_pack(__uint_as_float(s[2 * pi]), __uint_as_float(s[2 * pi + 1])), scale2, nbias2);
      y[hh] = ((kPolyPairs >> pi) & 1u) ? exp2_poly_pair(x) : exp2_mufu_pair(x);
    }
    l2a = add2(l2a, y[0]);
    l2b = add2(l2b, y[1]);
    float a, b, c, d;
    f32x2_unpack(y[0], a, b);
    f32x2_unpack(y[1], c, d);
    pw[w] = e4m3x2(a, b) | (e4m3x2(c, d) << 16);
  }
}
__device__ __forceinline__ float max_chunk(const uint32_t (&s)[32], float m) {
  float a = m, b = m;
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    a = max3(a, __uint_as_float(s[e]), __uint_as_float(s[e + 1]));
    b = max3(b, __uint_as_float(s[e + 2]), __uint_as_float(s[e + 3]));
  }
  return fmaxf(a, b);
}
__device__ __forceinline__ void mask_chunk(uint32_t (&s)[32], int valid) {
#pragma unroll
  for (int e = 0; e < 32; ++e)
    if (e >= valid) s[e] = __float_as_uint(-INFINITY);
}

template <int NT>
__global__ void __launch_bounds__(attn_threads(NT), 3 - NT)
    attn_fp8_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
  using L = AttnSmem<NT>;
  constexpr int kAttnStages = attn_stages(NT);
  constexpr int kProdWarp = 4 * NT, kMmaWarp = 4 * NT + 1;   // MMA warps kMmaWarp + tile
  constexpr uint32_t kTmemCols = 256 * NT, kOCol = 128 * NT;  // O of tile t at column kOCol + 128 t
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                // [stage]: K and V^T of a KV tile landed
  uint64_t* kv_empty = kv_full + kAttnStages;  // [stage]: both tiles' MMAs done reading it
  uint64_t* s_full = kv_empty + kAttnStages;   // [tile][half]: QK^T of the tile's current KV half landed
  // [tile][half]: P written over S by the tile's four softmax warps.  One barrier per S buffer: the softmax may
  // finish half i + 1 before the MMA warp waits for half i, which one barrier's phase parity could not tell apart.
  uint64_t* p_full = s_full + 4;
  uint64_t* pv_done = p_full + 4;              // [tile]: one phase per PV of a half
  uint64_t* o_done = pv_done + 2;              // [tile]: the tile's last PV done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const bool sparse = p.kv_ptr != nullptr;
  const int q0 = blockIdx.x * NT * kQTile;
  const bool has_b = NT == 2 && !sparse && q0 + kQTile < p.S;   // tile B holds queries of this sequence
  const int nkt = (p.S + 127) / 128;                  // KV tiles of the sequence
  // the CTA's KV steps: every KV tile in order (dense), or the query tile's list (block-sparse); step j reads KV tile
  // kvt_s[j] with K-block scale ksc_s[j].  An out-of-range list entry is recorded in the status word and skipped.
  int nkv = nkt;
  int kv0 = 0;
  if (sparse) {
    kv0 = p.kv_ptr[blockIdx.x];
    nkv = min(max(p.kv_ptr[blockIdx.x + 1] - kv0, 0), L::MAX_KBLK);
  }
  const int nhalf = 2 * nkv;
  float* ksc_s = reinterpret_cast<float*>(smem + L::KSC_OFF);
  int* kvt_s = reinterpret_cast<int*>(smem + L::KVT_OFF);
  for (int i = threadIdx.x; i < nkv; i += blockDim.x) {
    int kt = i;
    if (sparse) {
      kt = p.kv_idx[kv0 + i];
      if (kt < 0 || kt >= nkt) {
        set_status(220);
        kt = -1;
      }
    }
    kvt_s[i] = kt;
    ksc_s[i] = kt >= 0 ? p.kscale[(size_t)h * (p.SP / 128) + kt] : 0.f;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], has_b ? 2 : 1);   // one commit per MMA warp
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[2 * t], 1);
      mbar_init(&s_full[2 * t + 1], 1);
      mbar_init(&p_full[2 * t], 4);   // one arrival per softmax warp of the tile
      mbar_init(&p_full[2 * t + 1], 4);
      mbar_init(&pv_done[t], 1);
      mbar_init(&o_done[t], 1);
    }
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProdWarp) {
    // TMA producer: the whole warp runs the loop, one lane issues (warp-wide helpers)
    {
      if (lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
      }
      if (nkv > 0) {   // (nothing waits for Q when there is no KV step, so nothing is loaded)
        mbar_arrive_expect_tx(q_full, has_b ? 2 * L::TILE : L::TILE);
        tma_load_2d(smem + L::Q_OFF, &tmQ, 0, h * p.SP + q0, q_full);
        if (has_b) tma_load_2d(smem + L::Q_OFF + L::TILE, &tmQ, 0, h * p.SP + q0 + kQTile, q_full);
      }
      for (int j = 0; j < nkv; ++j) {
        const int st = j % kAttnStages;
        const uint32_t ph = (j / kAttnStages) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&kv_empty[st], ph ^ 1, 201))) break;
        uint8_t* kv = smem + L::KV_OFF + st * 2 * L::TILE;
        mbar_arrive_expect_tx(&kv_full[st], 2 * L::TILE);
        const int kt = max(kvt_s[j], 0);
        tma_load_2d(kv, &tmK, 0, h * p.SP + kt * 128, &kv_full[st]);
        tma_load_2d(kv + L::TILE, &tmV, kt * 128, h * 128, &kv_full[st]);
      }
    }
  } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
    const int t = warp - kMmaWarp;   // query tile this warp issues for (the whole warp; one lane issues)
    if (t == 0 || has_b) {
      constexpr uint32_t idesc_s = idesc_fp8(128, 64);
      constexpr uint32_t idesc_o = idesc_fp8(128, 128);
      const uint32_t qt = smem_u32(smem + L::Q_OFF + t * L::TILE);
      auto issue_s = [&](int i) {   // S_t[half] = Q_t K[keys of half i]^T (64 K rows = 8 KB into the K tile)
        const int hf = i & 1;
        const uint32_t ks = smem_u32(smem + L::KV_OFF + ((i >> 1) % kAttnStages) * 2 * L::TILE) + hf * 64 * 128;
#pragma unroll
        for (int kb = 0; kb < 4; ++kb)
          mma_fp8_ss(tmem + t * 128 + hf * 64, sdesc_kmajor_sw128(qt + kb * 32), sdesc_kmajor_sw128(ks + kb * 32),
                     idesc_s, kb != 0);
      };
      auto issue_pv = [&](int i) {   // O_t += P_t[half] V[keys of half i]
        const int hf = i & 1;
        const uint32_t vs = smem_u32(smem + L::KV_OFF + ((i >> 1) % kAttnStages) * 2 * L::TILE + L::TILE);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
          mma_fp8_ts(tmem + kOCol + t * 128, tmem + t * 128 + hf * 64 + kb * 32,
                     sdesc_kmajor_sw128(vs + (2 * hf + kb) * 32), idesc_o, (i | kb) != 0);
      };
      // (a query tile with no KV tile -- an empty block-sparse row -- issues nothing; its output rows are zero)
      bool ok = nhalf > 0 && __all_sync(0xffffffffu, mbar_wait(q_full, 0, 202) && mbar_wait(&kv_full[0], 0, 203));
      if (ok) {
        tc_fence_after();
        issue_s(0);
        tc_commit(&s_full[2 * t]);
        issue_s(1);
        tc_commit(&s_full[2 * t + 1]);
      }
      for (int i = 0; ok && i < nhalf; ++i) {
        const int hf = i & 1, j = i >> 1;
        const bool more = i + 2 < nhalf;
        // KV tile j + 1 normally lands long before P_t(i) does: wait for it first, so the MMAs follow P at once
        if (more && hf == 0 &&
            !(ok = __all_sync(0xffffffffu,
                              mbar_wait(&kv_full[(j + 1) % kAttnStages], ((j + 1) / kAttnStages) & 1, 206))))
          break;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&p_full[2 * t + hf], (i >> 1) & 1, 204 + t)))) break;
        tc_fence_after();
        issue_pv(i);
        tc_commit(&pv_done[t]);
        if (hf == 1) tc_commit(&kv_empty[j % kAttnStages]);
        if (more) {
          issue_s(i + 2);   // after PV_t(i) in issue order, so P_t(i) is consumed before S_t(i + 2) overwrites it
          tc_commit(&s_full[2 * t + hf]);
        }
      }
      tc_commit(&o_done[t]);
    }
  } else {
    // ------------------------------------------------------------------ softmax: one thread per query row
    const int t = warp >> 2;          // query tile
    const int qd = warp & 3;          // TMEM lane quadrant
    const int r = qd * 32 + lane;
    const int query = q0 + t * kQTile + r;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t o_col = tmem + lane_off + kOCol + t * 128;
    bool ok = t == 0 || has_b;
    const bool live = ok;
    const float qr = live ? p.qscale[(size_t)h * p.SP + query] : 0.f;
    float m_used = -INFINITY;
    uint64_t l2a = 0, l2b = 0;
    for (int i = 0; live && i < nhalf; ++i) {
      const int hf = i & 1;
      const uint32_t s_col = tmem + lane_off + t * 128 + hf * 64;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[2 * t + hf], (i >> 1) & 1, 210));
      if (!ok) break;
      tc_fence_after();
      uint32_t s0[32], s1[32];
      tmem_ld32(s_col, s0);
      tmem_ld32(s_col + 32, s1);
      tmem_ld_wait();
      // keys of this half inside the sequence (only the last KV tile is ragged; a skipped list entry has none)
      const int kt = kvt_s[i >> 1];
      const int valid = kt < 0 ? 0 : p.S - kt * 128 - hf * 64;
      if (valid < 64) {
        mask_chunk(s0, valid);
        mask_chunk(s1, valid - 32);
      }
      const float mx = fmaxf(max_chunk(s0, -INFINITY), max_chunk(s1, -INFINITY));
      const float scale = qr * ksc_s[i >> 1];
      const float mnew = mx * scale;
      // raise the running max only when the row's max grew by more than tau (then O and l are rescaled); a half
      // wholly past the sequence end has mx = -inf and changes nothing
      const bool need = mnew > m_used + kTau;
      float alpha = 1.0f;
      if (need) {
        alpha = ex2(m_used - mnew);
        m_used = mnew;
        const uint64_t a2 = f32x2_splat(alpha);
        l2a = mul2(l2a, a2);
        l2b = mul2(l2b, a2);
      }
      const uint64_t scale2 = f32x2_splat(scale), nbias2 = f32x2_splat(kPOffset - m_used);
      uint32_t pw[8];
      p_chunk(s0, scale2, nbias2, pw, l2a, l2b);
      tmem_st8(s_col, pw);
      p_chunk(s1, scale2, nbias2, pw, l2a, l2b);
      tmem_st8(s_col + 32, pw);
      // O must hold PV of every half < i before it is rescaled: wait for PV(i - 1) (issued when P(i - 1) was ready,
      // normally done by now; PV(i - 2) finished before S(i) was computed, so the phase parity is unambiguous).  The
      // tcgen05 ld/st are warp-wide, so a warp rescales when any of its rows must (the others multiply by 1).
      if (i > 0 && __any_sync(0xffffffffu, need)) {
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[t], (i - 1) & 1, 213));
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(o_col + 32 * c, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[2 * t + hf]);
    }
    // ---- epilogue: O / l * vscale -> bf16, this thread's row
    if (live) {
      ok = ok && mbar_wait(&o_done[t], 0, 212);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (live && ok) {
      tc_fence_after();
      float la, lb, lc, ld;
      f32x2_unpack(l2a, la, lb);
      f32x2_unpack(l2b, lc, ld);
      const float inv_l = nhalf > 0 ? 1.0f / ((la + lb) + (lc + ld)) : 0.0f;
      const float* vs = p.vscale + h * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(o_col + 32 * c, o);
        tmem_ld_wait();
        if (query < p.S) {
          __nv_bfloat16* orow = p.out + (long long)query * p.ldo;
          // to the token's owner's receive buffer (NVLink stores for other ranks' tokens).  No fence: whatever
          // reads them is ordered after this kernel's completion (a barrier on every rank), and a completed kernel's
          // writes, peer memory included, are visible to work ordered after it.
          if (p.ranks > 0) {
            const int owner = query / p.n_local;
            orow = reinterpret_cast<__nv_bfloat16*>(p.peer[owner]) +
                   (long long)(p.rank * p.n_local + query - owner * p.n_local) * p.ldo;
          }
          uint4* d4 = reinterpret_cast<uint4*>(orow + h * 128 + 32 * c);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              f[e] = nhalf > 0 ? __uint_as_float(o[q4 * 8 + e]) * inv_l * vs[32 * c + q4 * 8 + e] : 0.0f;
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
  if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace h3
