// HBM-bound kernels of the block: fused RMSNorm + adaLN modulation (+ NVFP4 quantisation), the standalone NVFP4
// quantiser, absmax, gated residual, activations, the modulation projection and the per-linear activation-scale
// state (dynamic / delayed scales).  Reference: tfvideo/kernels.py:15-84, tfvideo/linear.py:30-45,141-151,189-216,
// tfvideo/minimax_h3.py:265-269.
#pragma once

#include "common.cuh"
#include "h3b200.h"

namespace h3 {

// ------------------------------------------------------------------------------------------------ scale slots
// One slot per linear input (layout in h3b200.h): amax of this forward's input (-1 = none seen), the scale the
// quantiser uses (act), the delayed scale of the previous forward that was in use (used, 0 = none) and the margin.
__device__ __forceinline__ float slot_act(const H3ScaleSlot* s) { return s->act; }

// Dynamic scale of one call: act = max(amax, 1e-6) / 2688 (tfvideo/linear.py:148), float64 math held as fp32.
__global__ void act_from_amax_kernel(H3ScaleSlot* s) {
  double a = fmax((double)fmaxf(s->amax, 0.f), 1e-6) / 2688.0;
  s->act = (float)a;
}

// Begin a forward for n slots.  delayed = 0: every slot back to "no history" (tfvideo/linear.py:213-216).
// delayed = 1: tfvideo/linear.py:192-210 on the device: a slot whose input was seen last forward gets
// next = max(amax, 1e-6) / 2688 * margin, margin doubled (cap 16) if that input exceeded used * 2688; the new scale
// becomes this forward's act (and used).  `clipped` (nullable) receives the number of clipped slots.
__global__ void scales_begin_kernel(H3ScaleSlot* s, int n, int delayed, int* clipped) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  H3ScaleSlot v = s[i];
  if (!delayed) {
    v.amax = -1.f;
    v.act = 0.f;
    v.used = 0.f;
    v.margin = 0.f;
  } else if (v.amax >= 0.f) {
    double m = v.margin > 0.f ? (double)v.margin : 2.0;
    if (v.used > 0.f && (double)v.amax > (double)v.used * 2688.0) {
      m = fmin(m * 2.0, 16.0);
      if (clipped) atomicAdd(clipped, 1);
    }
    double nxt = fmax((double)v.amax, 1e-6) / 2688.0 * m;
    v.margin = (float)m;
    v.act = (float)nxt;
    v.used = (float)nxt;
    v.amax = -1.f;
  } else {
    v.used = 0.f;
  }
  s[i] = v;
}

// ------------------------------------------------------------------------------------------------ norm_mod
// One warp per row.  Lane l owns the 16-byte chunks at columns it * 256 + l * 8 (it < ceil(D / 256)); the sum of
// squares is accumulated per lane chunk by chunk (rounded product, rounded sum) and combined by an xor butterfly,
// so every lane holds the same bits; 1 / sqrt is an IEEE sqrt and an IEEE division.  oracle/ops.py:norm_mod states
// the same order, which makes the output (and the NVFP4 codes of it) bit-reproducible on the CPU.
// The row is read twice, once for the sum of squares and once for the transform; the second read hits L1 / L2.
// Holding the row in registers between the passes instead (80 registers a lane at D = 5120) left four warps per SM
// sub-partition, too few to cover the quantiser's dependent chains: 429 us against 253 us at S = 37,760.
struct NormModArgs {
  const __nv_bfloat16* x;
  int ldx;
  const float* w;
  const float* mod;
  const int* idx;
  int S, D, part;
  float eps;
  __nv_bfloat16* out;     // nullable: bf16 y
  int ldo;
  uint8_t* codes;         // nullable: NVFP4 codes [S, D/2]
  uint8_t* sf;            // scales, tiled (sf_tiled) or row-major [S, D/16]
  int sf_tiled;
  H3ScaleSlot* slot;      // nullable: amax of y is accumulated here; act is the quantiser's global scale
};

__global__ void __launch_bounds__(256) norm_mod_kernel(NormModArgs a) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= a.S) return;
  const int nit = (a.D + 255) >> 8;
  const __nv_bfloat16* xr = a.x + (size_t)row * a.ldx;
  float ss = 0.f;
#pragma unroll 4
  for (int it = 0; it < nit; ++it) {
    int c = it * 256 + lane * 8;
    if (c < a.D) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const uint32_t* w = &u.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float lo = bf16_lo(w[j]), hi = bf16_hi(w[j]);
        ss = __fadd_rn(ss, __fmul_rn(lo, lo));
        ss = __fadd_rn(ss, __fmul_rn(hi, hi));
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const float var = __fadd_rn(__fdiv_rn(ss, (float)a.D), a.eps);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(var));
  const size_t mrow = (size_t)a.idx[row] * 6 * a.D;
  const float* shift = a.mod + mrow + (size_t)(3 * a.part) * a.D;
  const float* scale = shift + a.D;
  float inv_g = 0.f;
  if (a.codes) inv_g = __fdiv_rn(1.0f, a.slot->act);
  float amax = 0.f;
  const int kgroups = a.D >> 4;
  const bool sf_words = (kgroups & 3) == 0;   // every 4-group quad lies inside the row
#pragma unroll 1
  for (int it = 0; it < nit; ++it) {
    int c = it * 256 + lane * 8;
    bool ok = c < a.D;
    float y[8];
    if (ok) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const uint32_t* wv = &u.x;
      float4 w0 = *reinterpret_cast<const float4*>(a.w + c), w1 = *reinterpret_cast<const float4*>(a.w + c + 4);
      float4 s0 = *reinterpret_cast<const float4*>(scale + c), s1 = *reinterpret_cast<const float4*>(scale + c + 4);
      float4 h0 = *reinterpret_cast<const float4*>(shift + c), h1 = *reinterpret_cast<const float4*>(shift + c + 4);
      const float wa[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const float sa[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      const float ha[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float xv = (j & 1) ? bf16_hi(wv[j >> 1]) : bf16_lo(wv[j >> 1]);
        float t = __fmul_rn(__fmul_rn(xv, r), wa[j]);
        t = __fadd_rn(__fmul_rn(t, __fadd_rn(1.0f, sa[j])), ha[j]);
        y[j] = bf16_round(t);
        amax = fmaxf(amax, fabsf(y[j]));
      }
      if (a.out) {
        uint4 o = make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]),
                             pack_bf16(y[6], y[7]));
        *reinterpret_cast<uint4*>(a.out + (size_t)row * a.ldo + c) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = 0.f;
    }
    if (a.codes) {
      // a 16-element group is the 8 values of lanes 2p and 2p+1
      float xs[8], gm = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xs[j] = __fmul_rn(y[j], inv_g);
        gm = fmaxf(gm, fabsf(xs[j]));
      }
      gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 1));
      uint32_t sfb = e4m3(div6_rn(gm));
      float inv = e4m3_rcp(sfb);
#pragma unroll
      for (int j = 0; j < 8; ++j) xs[j] = __fmul_rn(xs[j], inv);
      uint32_t cw = e2m1x8(xs);
      // the scales of groups 4b..4b+3 (lanes 8b, 8b+2, 8b+4, 8b+6) are 4 consecutive bytes in both layouts: one word
      const uint32_t w1 = __shfl_down_sync(0xffffffffu, sfb, 2), w2 = __shfl_down_sync(0xffffffffu, sfb, 4),
                     w3 = __shfl_down_sync(0xffffffffu, sfb, 6);
      if (ok) {
        *reinterpret_cast<uint32_t*>(a.codes + (size_t)row * (a.D >> 1) + (c >> 1)) = cw;
        const int k16 = c >> 4;
        const size_t off = a.sf_tiled ? sf_tiled_offset(row, k16, kgroups) : (size_t)row * kgroups + k16;
        if (sf_words) {
          if ((lane & 7) == 0) *reinterpret_cast<uint32_t*>(a.sf + off) = sfb | (w1 << 8) | (w2 << 16) | (w3 << 24);
        } else if ((lane & 1) == 0) {
          a.sf[off] = (uint8_t)sfb;
        }
      }
    }
  }
  if (a.slot) {
    amax = warp_max(amax);
    if (lane == 0) atomic_max_pos(&a.slot->amax, amax);
  }
}

// ------------------------------------------------------------------------------------------------ NVFP4 quantiser
// bf16 [R, K] -> NVFP4 (tfvideo/fp4attn.py:66-78 with a per-tensor scale, tfvideo/linear.py:30-38,148-151).  One
// thread per 16-element group.  The input element (r, c) is read at x + (c / cblk) * blk_stride + r * ldx + c % cblk,
// which also covers a row split into column blocks held apart (the Ulysses receive buffer); cblk = K for a plain
// matrix.  The global scale is *g_ptr when given, else g.  `amax` (nullable) receives max |x| (atomic).
struct QuantArgs {
  const __nv_bfloat16* x;
  long long ldx;
  int cblk;
  long long blk_stride;
  int R, K;
  const float* g_ptr;
  float g;
  uint8_t* codes;
  uint8_t* sf;
  int sf_tiled;
  float* amax;
};

__global__ void __launch_bounds__(256) nvfp4_quant_kernel(QuantArgs a) {
  const int groups = a.K >> 4;
  // the global scale's reciprocal once per block (one thread per group would otherwise divide per group)
  __shared__ float s_inv_g;
  if (threadIdx.x == 0) s_inv_g = __fdiv_rn(1.0f, a.g_ptr ? *a.g_ptr : a.g);
  __syncthreads();
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  float am = 0.f;
  uint32_t sfb = 0;
  size_t off = 0;
  const bool live = gid < (long long)a.R * groups;
  if (live) {
    const int r = (int)(gid / groups), k16 = (int)(gid % groups);
    const int c = k16 * 16;
    const __nv_bfloat16* src = a.x + (long long)(c / a.cblk) * a.blk_stride + (long long)r * a.ldx + (c % a.cblk);
    uint4 u0 = *reinterpret_cast<const uint4*>(src), u1 = *reinterpret_cast<const uint4*>(src + 8);
    const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    float v[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[2 * j] = bf16_lo(w[j]);
      v[2 * j + 1] = bf16_hi(w[j]);
      am = fmaxf(am, fmaxf(fabsf(v[2 * j]), fabsf(v[2 * j + 1])));
    }
    uint32_t cw[2];
    sfb = quant_group16(v, s_inv_g, cw);
    *reinterpret_cast<uint2*>(a.codes + (size_t)r * (a.K >> 1) + (c >> 1)) = make_uint2(cw[0], cw[1]);
    off = a.sf_tiled ? sf_tiled_offset(r, k16, groups) : (size_t)r * groups + k16;
    if ((groups & 3) != 0) a.sf[off] = (uint8_t)sfb;
  }
  // with groups % 4 == 0, lanes 4b..4b+3 hold the scales of 4 consecutive groups of one row: one word store
  if ((groups & 3) == 0) {
    const uint32_t w1 = __shfl_down_sync(0xffffffffu, sfb, 1), w2 = __shfl_down_sync(0xffffffffu, sfb, 2),
                   w3 = __shfl_down_sync(0xffffffffu, sfb, 3);
    if (live && (threadIdx.x & 3) == 0)
      *reinterpret_cast<uint32_t*>(a.sf + off) = sfb | (w1 << 8) | (w2 << 16) | (w3 << 24);
  }
  if (a.amax) {
    am = warp_max(am);
    if ((threadIdx.x & 31) == 0) atomic_max_pos(a.amax, am);
  }
}

// max |x| over a bf16 [R, K] matrix (row stride ldx), atomically into *out (tfvideo/linear.py:41-45).
__global__ void __launch_bounds__(256) absmax_kernel(const __nv_bfloat16* x, long long ldx, int R, int K, float* out) {
  float am = 0.f;
  const int vec = K >> 3;
  const long long n = (long long)R * vec;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / vec, c = (i % vec) * 8;
    uint4 u = *reinterpret_cast<const uint4*>(x + r * ldx + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) am = fmaxf(am, fmaxf(fabsf(bf16_lo(w[j])), fabsf(bf16_hi(w[j]))));
  }
  am = warp_max(am);
  if ((threadIdx.x & 31) == 0) atomic_max_pos(out, am);
}

// ------------------------------------------------------------------------------------------------ gate_add
// x += y * gate[idx] in place, bf16 (tfvideo/kernels.py:43-63); rounded product then rounded sum.
__global__ void __launch_bounds__(256) gate_add_kernel(__nv_bfloat16* x, int ldx, const __nv_bfloat16* y, int ldy,
                                                       const float* mod, const int* idx, int S, int D, int part) {
  const int vec = D >> 3;
  const long long n = (long long)S * vec;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    int r = (int)(i / vec), c = (int)(i % vec) * 8;
    const float* g = mod + ((size_t)idx[r] * 6 + 3 * part + 2) * D + c;
    float4 g0 = *reinterpret_cast<const float4*>(g), g1 = *reinterpret_cast<const float4*>(g + 4);
    const float ga[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    uint4* xp = reinterpret_cast<uint4*>(x + (size_t)r * ldx + c);
    uint4 xu = *xp, yu = *reinterpret_cast<const uint4*>(y + (size_t)r * ldy + c);
    uint32_t* xw = &xu.x;
    const uint32_t* yw = &yu.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float lo = __fadd_rn(bf16_lo(xw[j]), __fmul_rn(bf16_lo(yw[j]), ga[2 * j]));
      float hi = __fadd_rn(bf16_hi(xw[j]), __fmul_rn(bf16_hi(yw[j]), ga[2 * j + 1]));
      xw[j] = pack_bf16(lo, hi);
    }
    *xp = xu;
  }
}

// ------------------------------------------------------------------------------------------------ activations
__device__ __forceinline__ float gelu_tanh_f(float u) {
  // 0.5 u (1 + tanh(z)) with z = sqrt(2/pi) (u + 0.044715 u^3), evaluated as u * sigmoid(2 z) = u / (1 + e^(-2z)):
  // the same function without the cancellation of 1 + tanh(z) for negative z
  const float z2 = 1.5957691216057308f * (u + 0.044715f * u * u * u);
  return __fdividef(u, 1.0f + __expf(-z2));
}
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// act = gelu_tanh(u) (act_kind 0, u [M, F]) or silu(gate) * up (act_kind 1, u = [gate | up] [M, 2F]); bf16 out
// [M, F].  `amax` (nullable) receives max |act|.  tfvideo/kernels.py:66-84.
__global__ void __launch_bounds__(256) act_kernel(const __nv_bfloat16* u, int ldu, __nv_bfloat16* out, int ldo, int M,
                                                  int F, int act_kind, float* amax) {
  const int vec = F >> 3;
  const long long n = (long long)M * vec;
  float am = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    int r = (int)(i / vec), c = (int)(i % vec) * 8;
    uint4 a = *reinterpret_cast<const uint4*>(u + (size_t)r * ldu + c);
    uint4 b = act_kind ? *reinterpret_cast<const uint4*>(u + (size_t)r * ldu + F + c) : a;
    const uint32_t* aw = &a.x;
    const uint32_t* bw = &b.x;
    uint4 o;
    uint32_t* ow = &o.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float lo, hi;
      if (act_kind) {
        lo = silu_mul(bf16_lo(aw[j]), bf16_lo(bw[j]));
        hi = silu_mul(bf16_hi(aw[j]), bf16_hi(bw[j]));
      } else {
        lo = gelu_tanh_f(bf16_lo(aw[j]));
        hi = gelu_tanh_f(bf16_hi(aw[j]));
      }
      ow[j] = pack_bf16(lo, hi);
      am = fmaxf(am, fmaxf(fabsf(bf16_lo(ow[j])), fabsf(bf16_hi(ow[j]))));
    }
    *reinterpret_cast<uint4*>(out + (size_t)r * ldo + c) = o;
  }
  if (amax) {
    am = warp_max(am);
    if ((threadIdx.x & 31) == 0) atomic_max_pos(amax, am);
  }
}

// ------------------------------------------------------------------------------------------------ modulation
// mod[m, j] = ada_b[j] + sum_t t_emb[m, t] * ada_w[j, t], fp32, [M, 18 D] (viewed [3M, 6, D]); tfvideo/minimax_h3.py:265-269.
__global__ void __launch_bounds__(256) modulation_kernel(const float* t_emb, int M, int t_dim, const float* ada_w,
                                                         const float* ada_b, int J, float* mod) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)M * J) return;
  int m = (int)(i / J), j = (int)(i % J);
  const float* w = ada_w + (size_t)j * t_dim;
  const float* t = t_emb + (size_t)m * t_dim;
  float acc = 0.f;
  for (int k = 0; k < t_dim; ++k) acc = fmaf(t[k], w[k], acc);
  mod[i] = ada_b[j] + acc;
}

}  // namespace h3
