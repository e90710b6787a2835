// NVFP4 W4A4 GEMM for sm_100a: D[M, N] = (A_codes * sfA * gA) x (B_codes * sfB * gB)^T with block-scaled tcgen05 MMAs
// (kind::mxf4nvf4, one UE4M3 scale per 16 elements), fp32 accumulators in TMEM, A/B tiles fed by TMA and the scale
// tiles by bulk copies, and the block's elementwise work fused into the epilogue.  It replaces the reference's
// Nvfp4Linear.__call__ -> TensorFold prompt(A4, x, lin) (tfvideo/linear.py:141-151) and, through the epilogues,
// kernels.gate_add (tfvideo/kernels.py:43-63) and the activation + requantisation of fc1
// (tfvideo/kernels.py:66-84, tfvideo/linear.py:219-233).
//
// CTA tile 128 x BN (BN = 256 or 128), K tile 256 elements (128 bytes, one 128-byte swizzle row), 4-stage smem ring.
// Warp 0: TMA producer.  Warp 1: TMEM owner and MMA issuer (one thread).  Warps 2-5: epilogue, warp w reading TMEM
// lanes 32 * (w % 4) .. +31, i.e. one output row per thread.
#pragma once

#include "common.cuh"
#include "h3b200.h"

namespace h3 {

struct GemmArgs {
  const uint8_t* sfa;            // tiled scales of A, ceil(M/128) * 128 rows x K/16
  const uint8_t* sfb;            // tiled scales of B, N rows x K/16
  int M, N, K;
  const H3ScaleSlot* a_slot;     // act of A's quantisation (global scale gA)
  float g_b;                     // global scale of B
  const float* bias;             // nullable, fp32 [N]
  int epi;                       // H3_EPI_*
  __nv_bfloat16* out;            // STORE / ACT_BF16 output (ACT_Q: optional copy of the activation)
  long long ldo;
  __nv_bfloat16* x;              // GATE_RESID residual, updated in place
  long long ldx;
  const float* mod;              // [R, 6, N] modulation rows
  const int* idx;                // [M] modulation row of each row
  int gate_part;                 // 0: chunk 2 (gate_msa), 1: chunk 5 (gate_mlp)
  int act_kind;                  // 0: gelu_tanh, 1: swiglu on 16-column interleaved [gate | up]
  uint8_t* qcodes;               // ACT_Q: NVFP4 codes of the activation [M, F/2]
  uint8_t* qsf;                  // ACT_Q: tiled scales of the activation
  H3ScaleSlot* q_slot;           // ACT_BF16 / ACT_Q: amax of the activation; ACT_Q quantises under q_slot->act
};

constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;

template <int BN>
struct GemmSmem {
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int SFA_BYTES = 2048;
  static constexpr int SFB_BYTES = (BN / 128) * 2048;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  static constexpr int BAR_OFF = kGemmStages * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;     // barriers + TMEM address word + alignment slack
  // TMEM columns: accumulator [0, BN), then one scale-factor buffer per smem stage: A scales (4 columns per MMA K
  // step, 4 steps) and B scales (BN / 32 per K step).  A K-tile's copies go to its own buffer, so they never wait for
  // the previous K-tile's MMAs to finish reading theirs.
  static constexpr int SF_COLS = 16 + BN / 8;
  static constexpr int SFA_COL = BN;
  static constexpr int SFB_COL = BN + 16;
  static constexpr int TMEM_COLS = 512;
  static_assert(BN + kGemmStages * SF_COLS <= TMEM_COLS, "TMEM budget");
};

__device__ __forceinline__ float act_apply(int kind, float g, float u) {
  return kind ? silu_mul(g, u) : gelu_tanh_f(u);
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs p) {
  using L = GemmSmem<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + kGemmStages;
  uint64_t* acc_full = empty + kGemmStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m_blk = blockIdx.y, m0 = m_blk * 128;
  const int KT = p.K >> 8;
  const int kblocks64 = p.K >> 6;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % kGemmStages;
        const uint32_t ph = (kt / kGemmStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, 101)) break;
        uint8_t* st = smem + s * L::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
        tma_load_2d(st, &tmA, kt * 128, m0, &full[s]);
        tma_load_2d(st + L::A_BYTES, &tmB, kt * 128, n0, &full[s]);
        bulk_load(st + L::A_BYTES + L::B_BYTES, p.sfa + ((size_t)m_blk * kblocks64 + kt * 4) * 512, 2048, &full[s]);
#pragma unroll
        for (int nb = 0; nb < BN / 128; ++nb)
          bulk_load(st + L::A_BYTES + L::B_BYTES + L::SFA_BYTES + nb * 2048,
                    p.sfb + ((size_t)(n0 / 128 + nb) * kblocks64 + kt * 4) * 512, 2048, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_nvfp4(128, BN);
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % kGemmStages;
        const uint32_t ph = (kt / kGemmStages) & 1;
        if (!mbar_wait(&full[s], ph, 102)) break;
        tc_fence_after();
        uint8_t* st = smem + s * L::STAGE_BYTES;
        const uint32_t a_s = smem_u32(st), b_s = smem_u32(st + L::A_BYTES);
        const uint32_t sfa_s = smem_u32(st + L::A_BYTES + L::B_BYTES);
        const uint32_t sfb_s = sfa_s + L::SFA_BYTES;
        const uint32_t sf_t = tmem + s * L::SF_COLS;   // this stage's scale-factor buffer
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          tmem_cp_32x128b_x4(sf_t + L::SFA_COL + 4 * kb, sdesc_sf_atom(sfa_s + kb * 512));
#pragma unroll
          for (int nb = 0; nb < BN / 128; ++nb)
            tmem_cp_32x128b_x4(sf_t + L::SFB_COL + (BN / 32) * kb + 4 * nb, sdesc_sf_atom(sfb_s + nb * 2048 + kb * 512));
        }
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          mma_nvfp4(tmem, sdesc_kmajor_sw128(a_s + kb * 32), sdesc_kmajor_sw128(b_s + kb * 32), idesc,
                    sf_t + L::SFA_COL + 4 * kb, sf_t + L::SFB_COL + (BN / 32) * kb, (kt | kb) != 0);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const bool live = row < p.M;
    __nv_bfloat16* __restrict__ xrow = nullptr;
    const float* __restrict__ gate = nullptr;
    if (p.epi == H3_EPI_GATE_RESID && live) {
      // the residual tile is read after the mainloop: pull this row's 2 * BN bytes into L2 while the MMAs run
      xrow = p.x + (size_t)row * p.ldx + n0;
      gate = p.mod + ((size_t)p.idx[row] * 6 + 3 * p.gate_part + 2) * p.N + n0;
#pragma unroll
      for (int b = 0; b < BN * 2; b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"((const char*)xrow + b));
    }
    const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, 103));   // tcgen05.ld below is warp-wide
    tc_fence_after();
    if (ok) {
      const float alpha = p.a_slot->act * p.g_b;
      float inv_q = 0.f;
      if (p.epi == H3_EPI_ACT_Q) inv_q = __fdiv_rn(1.0f, p.q_slot->act);
      float amax = 0.f;
      const int F = p.act_kind ? (p.N >> 1) : p.N;   // activation width (ACT_*)
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        // issue this chunk's global loads (residual, gate) before the TMEM load so their latency overlaps it
        uint4 xu[4];
        float4 ga[8];
        if (xrow) {
#pragma unroll
          for (int j = 0; j < 4; ++j) xu[j] = reinterpret_cast<const uint4*>(xrow + c * 32)[j];
#pragma unroll
          for (int j = 0; j < 8; ++j) ga[j] = reinterpret_cast<const float4*>(gate + c * 32)[j];
        }
        __syncwarp();
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, r);
        tmem_ld_wait();
        const int nc = n0 + c * 32;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] = __uint_as_float(r[j]) * alpha;
          if (p.bias) v[j] += p.bias[nc + j];
        }
        if (!live) continue;
        if (p.epi == H3_EPI_STORE) {
          uint4* o = reinterpret_cast<uint4*>(p.out + (size_t)row * p.ldo + nc);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            o[j] = make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                              pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
        } else if (p.epi == H3_EPI_GATE_RESID) {
          const float* g = reinterpret_cast<const float*>(ga);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t* xw = &xu[j].x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int k = 8 * j + 2 * e;
              float lo = __fadd_rn(bf16_lo(xw[e]), __fmul_rn(bf16_round(v[k]), g[k]));
              float hi = __fadd_rn(bf16_hi(xw[e]), __fmul_rn(bf16_round(v[k + 1]), g[k + 1]));
              xw[e] = pack_bf16(lo, hi);
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(xrow + c * 32)[j] = xu[j];
        } else {
          // activation: gelu -> 32 outputs at columns nc.., swiglu -> 16 outputs at columns nc / 2..
          float a[32];
          const int na = p.act_kind ? 16 : 32;
          const int fc = p.act_kind ? (nc >> 1) : nc;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < na) {
              float y = p.act_kind ? act_apply(1, bf16_round(v[j]), bf16_round(v[j + 16]))
                                   : act_apply(0, 0.f, bf16_round(v[j]));
              a[j] = bf16_round(y);
              amax = fmaxf(amax, fabsf(a[j]));
            } else {
              a[j] = 0.f;
            }
          }
          if (p.out) {
            uint4* o = reinterpret_cast<uint4*>(p.out + (size_t)row * p.ldo + fc);
            for (int j = 0; j < na / 8; ++j)
              o[j] = make_uint4(pack_bf16(a[8 * j], a[8 * j + 1]), pack_bf16(a[8 * j + 2], a[8 * j + 3]),
                                pack_bf16(a[8 * j + 4], a[8 * j + 5]), pack_bf16(a[8 * j + 6], a[8 * j + 7]));
          }
          if (p.epi == H3_EPI_ACT_Q) {
            const int kgroups = F >> 4;
            for (int gi = 0; gi < na / 16; ++gi) {
              float g16[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) g16[e] = a[gi * 16 + e];
              uint32_t cw[2];
              uint32_t sfb = quant_group16(g16, inv_q, cw);
              const int col = fc + gi * 16;
              *reinterpret_cast<uint2*>(p.qcodes + (size_t)row * (F >> 1) + (col >> 1)) = make_uint2(cw[0], cw[1]);
              p.qsf[sf_tiled_offset(row, col >> 4, kgroups)] = (uint8_t)sfb;
            }
          }
        }
      }
      if (p.q_slot && (p.epi == H3_EPI_ACT_BF16 || p.epi == H3_EPI_ACT_Q)) {
        amax = warp_max(amax);
        if (lane == 0) atomic_max_pos(&p.q_slot->amax, amax);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, L::TMEM_COLS);
}

}  // namespace h3
