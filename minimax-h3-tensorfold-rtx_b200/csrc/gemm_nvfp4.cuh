// NVFP4 W4A4 GEMM for sm_100a: D[M, N] = (A_codes * sfA * gA) x (B_codes * sfB * gB)^T with block-scaled tcgen05 MMAs
// (kind::mxf4nvf4, one UE4M3 scale per 16 elements), fp32 accumulators in TMEM, A/B tiles fed by TMA and the scale
// tiles by bulk copies, and the block's elementwise work fused into the epilogue.  It replaces the reference's
// Nvfp4Linear.__call__ -> TensorFold prompt(A4, x, lin) (tfvideo/linear.py:141-151) and, through the epilogues,
// kernels.gate_add (tfvideo/kernels.py:43-63) and the activation + requantisation of fc1
// (tfvideo/kernels.py:66-84, tfvideo/linear.py:219-233).
//
// CTA tile 128 x BN (BN = 256 or 128), K tile 256 elements (128 bytes, one 128-byte swizzle row), 4-stage smem ring.
// Warp 0: TMA producer.  Warp 1: TMEM owner and MMA issuer (one thread).  Warps 2..: epilogue, warp w reading TMEM
// lanes 32 * (w % 4) .. +31 (one output row per thread) and share (w - 2) / 4 of the columns.  Persistent over tiles.
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
  // STORE_PEERS: the qkv rows of this rank's M tokens, each head's 128 columns to the rank owning the head
  unsigned long long peer[8];
  int ranks, rank;
};

constexpr int kGemmStages = 4;
// Warp 0 TMA, warp 1 MMA, then the epilogue warps: kGemmEpiWarps(EPI) per TMEM lane quadrant.  The activation
// epilogues (GELU / SwiGLU + NVFP4 requantisation) do several times the arithmetic of the others per element and
// take four, so that one tile's epilogue stays shorter than the next tile's mainloop.
__host__ __device__ constexpr int kGemmEpiWarps(int epi) { return (epi == H3_EPI_ACT_Q || epi == H3_EPI_ACT_BF16) ? 4 : 2; }
__host__ __device__ constexpr int kGemmThreads(int epi) { return 64 + 128 * kGemmEpiWarps(epi); }

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

// Persistent: grid = min(#tiles, #SMs) CTAs walk the tiles round-robin (tile t -> m block t / tiles_n, n block
// t % tiles_n, so the CTAs in flight share A rows and stream B through L2).  One accumulator in TMEM: the epilogue
// warps first copy it out as packed bf16 (every epilogue rounds y to bf16 first) and hand TMEM back to the MMA warp,
// then do the global-memory half of the epilogue while the next tile's MMAs run.
// The 16 packed words (32 bf16 values) of chunk c of the staged accumulator row; a switch keeps `hold` in registers
// while the chunk loop itself stays rolled (small code for the heavy epilogues).
template <int K, int N>
__device__ __forceinline__ void copy_chunk(const uint32_t (&hold)[N], uint32_t (&y)[16]) {
  if constexpr (K < N / 16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = hold[K * 16 + j];
  }
}
template <int N>
__device__ __forceinline__ void chunk_words(const uint32_t (&hold)[N], int c, uint32_t (&y)[16]) {
  switch (c) {
    case 0: copy_chunk<0>(hold, y); break;
    case 1: copy_chunk<1>(hold, y); break;
    case 2: copy_chunk<2>(hold, y); break;
    case 3: copy_chunk<3>(hold, y); break;
    case 4: copy_chunk<4>(hold, y); break;
    case 5: copy_chunk<5>(hold, y); break;
    case 6: copy_chunk<6>(hold, y); break;
    default: copy_chunk<7>(hold, y); break;
  }
}

// ---- epilogue pieces shared by the 1-CTA and the CTA-pair kernels
// Phase 1: the CW accumulator columns [cofs, cofs + CW) of this thread's row (TMEM lane quadrant q) -> packed
// bf16(acc * alpha + bias[ncol0 + ...]) in registers.  Every epilogue rounds y to bf16 first.
template <int CW>
__device__ __forceinline__ void epi_load(uint32_t (&hold)[CW / 2], uint32_t tmem, int q, int cofs, int ncol0,
                                         float alpha, const float* __restrict__ bias) {
#pragma unroll
  for (int c = 0; c < CW / 32; ++c) {
    uint32_t r[32];
    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + cofs + c * 32, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v0 = __uint_as_float(r[2 * j]) * alpha, v1 = __uint_as_float(r[2 * j + 1]) * alpha;
      if (bias) {
        v0 += bias[ncol0 + c * 32 + 2 * j];
        v1 += bias[ncol0 + c * 32 + 2 * j + 1];
      }
      hold[c * 16 + j] = pack_bf16(v0, v1);
    }
  }
}

// Phase 2: the fused consumer of row `row`'s CW columns starting at global column n0c (held as packed bf16), in
// 32-column chunks: a store (to this rank's output or, STORE_PEERS, to the owner of each head), the gated residual
// (xrow / gate: this row's slices of x and of the gate row), or the activation with its amax and NVFP4 codes.
template <int EPI, int CW>
__device__ __forceinline__ void epi_store(const GemmArgs& p, const uint32_t (&hold)[CW / 2], int row, int n0c,
                                          __nv_bfloat16* __restrict__ xrow, const float* __restrict__ gate,
                                          float inv_q, int F, float& amax) {
#pragma unroll 1
  for (int c = 0; c < CW / 32; ++c) {
    const int nc = n0c + c * 32;
    uint32_t y[16];   // 32 bf16 values, columns nc..nc+31
    chunk_words(hold, c, y);
    if (EPI == H3_EPI_STORE || EPI == H3_EPI_STORE_PEERS) {
      __nv_bfloat16* dst = p.out + (size_t)row * p.ldo + nc;
      if (EPI == H3_EPI_STORE_PEERS) {
        // column nc = (part, head, d): a 32-column chunk lies inside one 128-column head
        const int H = p.N / 384, Hr = H / p.ranks;
        const int part = nc / (H * 128), head = (nc >> 7) - part * H, d = nc & 127;
        const int owner = head / Hr;
        dst = reinterpret_cast<__nv_bfloat16*>(p.peer[owner]) +
              ((size_t)((p.rank * p.M + row) * 3 + part) * Hr + (head - owner * Hr)) * 128 + d;
      }
      uint4* o = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = make_uint4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
    } else if (EPI == H3_EPI_GATE_RESID) {
      uint4 xu[4];
      float4 ga[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) xu[j] = reinterpret_cast<const uint4*>(xrow + c * 32)[j];
#pragma unroll
      for (int j = 0; j < 8; ++j) ga[j] = reinterpret_cast<const float4*>(gate + c * 32)[j];
      const float* g = reinterpret_cast<const float*>(ga);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t* xw = &xu[j].x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 8 * j + 2 * e;
          const uint32_t yw = y[k >> 1];
          float lo = __fadd_rn(bf16_lo(xw[e]), __fmul_rn(bf16_lo(yw), g[k]));
          float hi = __fadd_rn(bf16_hi(xw[e]), __fmul_rn(bf16_hi(yw), g[k + 1]));
          xw[e] = pack_bf16(lo, hi);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(xrow + c * 32)[j] = xu[j];
    } else {
      // activation, one 16-wide NVFP4 group at a time: gelu -> groups at columns nc, nc + 16;
      // swiglu (16-column interleaved [gate | up]) -> one group at column nc / 2
      const int ngroups = p.act_kind ? 1 : 2;
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        if (gi >= ngroups) break;
        const int col = (p.act_kind ? (nc >> 1) : nc) + gi * 16;
        float a16[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int j = gi * 16 + e;
          const float u = (j & 1) ? bf16_hi(y[j >> 1]) : bf16_lo(y[j >> 1]);
          float av;
          if (p.act_kind) {
            const uint32_t uw = y[(e + 16) >> 1];
            av = act_apply(1, u, (e & 1) ? bf16_hi(uw) : bf16_lo(uw));
          } else {
            av = act_apply(0, 0.f, u);
          }
          a16[e] = bf16_round(av);
          amax = fmaxf(amax, fabsf(a16[e]));
        }
        if (p.out) {
          uint4* o = reinterpret_cast<uint4*>(p.out + (size_t)row * p.ldo + col);
          o[0] = make_uint4(pack_bf16(a16[0], a16[1]), pack_bf16(a16[2], a16[3]), pack_bf16(a16[4], a16[5]),
                            pack_bf16(a16[6], a16[7]));
          o[1] = make_uint4(pack_bf16(a16[8], a16[9]), pack_bf16(a16[10], a16[11]), pack_bf16(a16[12], a16[13]),
                            pack_bf16(a16[14], a16[15]));
        }
        if (EPI == H3_EPI_ACT_Q) {
          uint32_t cw[2];
          const uint32_t sfb = quant_group16(a16, inv_q, cw);
          *reinterpret_cast<uint2*>(p.qcodes + (size_t)row * (F >> 1) + (col >> 1)) = make_uint2(cw[0], cw[1]);
          p.qsf[sf_tiled_offset(row, col >> 4, F >> 4)] = (uint8_t)sfb;
        }
      }
    }
  }
}

// This thread's slices of x and of the gate row for the gated-residual epilogue, pulled into L2 while the tile's MMAs
// run (other epilogues: null).
template <int EPI, int CW>
__device__ __forceinline__ void epi_prefetch(const GemmArgs& p, int row, int n0c, __nv_bfloat16*& xrow,
                                             const float*& gate) {
  xrow = nullptr;
  gate = nullptr;
  if (EPI == H3_EPI_GATE_RESID && row < p.M) {
    xrow = p.x + (size_t)row * p.ldx + n0c;
    gate = p.mod + ((size_t)p.idx[row] * 6 + 3 * p.gate_part + 2) * p.N + n0c;
#pragma unroll
    for (int b = 0; b < 2 * CW; b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"((const char*)xrow + b));
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads(EPI), 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs p) {
  using L = GemmSmem<BN>;
  constexpr int EW = kGemmEpiWarps(EPI);   // epilogue warps per lane quadrant
  constexpr int CW = BN / EW;              // columns of one epilogue thread
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + kGemmStages;
  uint64_t* acc_full = empty + kGemmStages;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = p.K >> 8;
  const int kblocks64 = p.K >> 6;
  const int tiles_n = p.N / BN;
  const int tiles = ((p.M + 127) >> 7) * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4 * EW);
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
    // ------------------------------------------------------------------ TMA producer (the whole warp; one lane issues)
    {
      if (lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
      }
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int m_blk = t / tiles_n, n0 = (t % tiles_n) * BN;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % kGemmStages;
          const uint32_t ph = (it / kGemmStages) & 1;
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, 101)))) break;
          uint8_t* st = smem + s * L::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
          tma_load_2d(st, &tmA, kt * 128, m_blk * 128, &full[s]);
          tma_load_2d(st + L::A_BYTES, &tmB, kt * 128, n0, &full[s]);
          bulk_load(st + L::A_BYTES + L::B_BYTES, p.sfa + ((size_t)m_blk * kblocks64 + kt * 4) * 512, 2048,
                    &full[s]);
#pragma unroll
          for (int nb = 0; nb < BN / 128; ++nb)
            bulk_load(st + L::A_BYTES + L::B_BYTES + L::SFA_BYTES + nb * 2048,
                      p.sfb + ((size_t)(n0 / 128 + nb) * kblocks64 + kt * 4) * 512, 2048, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (the whole warp; one lane issues)
    {
      constexpr uint32_t idesc = idesc_nvfp4(128, BN);
      uint32_t it = 0, ti = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++ti) {
        if (ti > 0 && !(ok = __all_sync(0xffffffffu, mbar_wait(acc_empty, (ti - 1) & 1, 104)))) break;
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % kGemmStages;
          const uint32_t ph = (it / kGemmStages) & 1;
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ph, 102)))) break;
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
              tmem_cp_32x128b_x4(sf_t + L::SFB_COL + (BN / 32) * kb + 4 * nb,
                                 sdesc_sf_atom(sfb_s + nb * 2048 + kb * 512));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb)
            mma_nvfp4(tmem, sdesc_kmajor_sw128(a_s + kb * 32), sdesc_kmajor_sw128(b_s + kb * 32), idesc,
                      sf_t + L::SFA_COL + 4 * kb, sf_t + L::SFB_COL + (BN / 32) * kb, (kt | kb) != 0);
          tc_commit(&empty[s]);
        }
        tc_commit(acc_full);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int cofs = ((warp - 2) >> 2) * CW;   // this warp's share of the tile's columns
    const float alpha = p.a_slot->act * p.g_b;
    const float inv_q = EPI == H3_EPI_ACT_Q ? __fdiv_rn(1.0f, p.q_slot->act) : 0.f;
    const int F = p.act_kind ? (p.N >> 1) : p.N;   // activation width (ACT_*)
    float amax = 0.f;
    uint32_t ti = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++ti) {
      const int m_blk = t / tiles_n, n0 = (t % tiles_n) * BN;
      const int row = m_blk * 128 + q * 32 + lane;
      const bool live = row < p.M;
      __nv_bfloat16* xrow;
      const float* gate;
      epi_prefetch<EPI, CW>(p, row, n0 + cofs, xrow, gate);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, ti & 1, 103));   // tcgen05.ld is warp-wide
      if (!ok) break;
      tc_fence_after();
      // phase 1: accumulator -> registers, then TMEM goes back to the MMA warp; phase 2 overlaps the next tile
      uint32_t hold[CW / 2];
      epi_load<CW>(hold, tmem, q, cofs, n0 + cofs, alpha, p.bias);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      if (!live) continue;
      epi_store<EPI, CW>(p, hold, row, n0 + cofs, xrow, gate, inv_q, F, amax);
    }
    if (p.q_slot && (EPI == H3_EPI_ACT_BF16 || EPI == H3_EPI_ACT_Q)) {
      amax = warp_max(amax);
      if (lane == 0) atomic_max_pos(&p.q_slot->amax, amax);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, L::TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------ CTA-pair GEMM
// The same GEMM on CTA pairs (a cluster of two CTAs on two SMs, tcgen05 cta_group::2): one 256 x 256 output tile per
// pair, each CTA holding 128 of its rows.  Per 256-element K tile a CTA loads its 128 rows of A and its 128 of the
// tile's 256 B rows (the pair's MMA reads the other CTA's half), plus the scales of its A rows and of all 256 B rows:
// 38 KB against the 54 KB a 128 x 256 tile needs alone, so a third less L2 traffic per FLOP and five stages in flight
// instead of four.  The leader (rank 0) issues the scale copies and the MMAs of the pair; both CTAs' TMA loads count
// on the leader's stage barriers; the leader's commits release the stage and hand over the accumulator in both CTAs;
// both CTAs' epilogues (the same code as the 1-CTA kernel) return the accumulator to the leader.  No load
// multicasts: every CTA loads its own data.  Used when N % 256 == 0.
struct GemmPairSmem {
  static constexpr int A_BYTES = 128 * 128;       // 128 rows x 256 K elements of NVFP4 codes
  static constexpr int B_BYTES = 128 * 128;       // this CTA's 128 of the tile's 256 B rows
  static constexpr int SFA_BYTES = 2048;          // scales of this CTA's 128 A rows
  static constexpr int SFB_BYTES = 4096;          // scales of all 256 B rows: each CTA's half of the MMA needs them
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;   // 38 KB (a multiple of 1024)
  static constexpr int STAGES = 5;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
  // TMEM: accumulator [0, 256), then per stage the A scales (4 columns a K step) and the B scales (8 a K step)
  static constexpr int SF_COLS = 16 + 32;
  static constexpr int TMEM_COLS = 512;
  static_assert(256 + STAGES * SF_COLS <= TMEM_COLS, "TMEM budget");
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment for the swizzled tiles");
};

template <int EPI>
__global__ void __launch_bounds__(kGemmThreads(EPI), 1)
    gemm_nvfp4_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB,
                           const GemmArgs p) {
  using L = GemmPairSmem;
  constexpr int BN = 256;
  constexpr int EW = kGemmEpiWarps(EPI);
  constexpr int CW = BN / EW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);   // [stage] (the leader's are the ones used)
  uint64_t* empty = full + L::STAGES;                                 // [stage] (each CTA's own)
  uint64_t* acc_full = empty + L::STAGES;
  uint64_t* acc_empty = acc_full + 1;                                 // the leader's counts both CTAs' epilogues
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int KT = p.K >> 8;
  const int tiles_n = p.N / BN;
  const int tiles = ((p.M + 255) >> 8) * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * 4 * EW);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, L::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();   // both CTAs' barriers initialised (the peer's loads land on the leader's) and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      prefetch_tmap(&tmSA);
      prefetch_tmap(&tmSB);
    }
    uint32_t it = 0;
    bool ok = true;
    for (int t = pair; ok && t < tiles; t += npairs) {
      const int m_blk = t / tiles_n, n_blk = t % tiles_n;
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % L::STAGES;
        const uint32_t ph = (it / L::STAGES) & 1;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, 111)))) break;
        if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * L::STAGE_BYTES);   // the pair's bytes of this stage
        const uint32_t bar = cluster_addr(&full[s], 0);
        uint8_t* st = smem + s * L::STAGE_BYTES;
        tma_load_2d_pair(st, &tmA, kt * 128, m_blk * 256 + (int)rank * 128, bar);
        tma_load_2d_pair(st + L::A_BYTES, &tmB, kt * 128, n_blk * 256 + (int)rank * 128, bar);
        tma_load_2d_pair(st + L::A_BYTES + L::B_BYTES, &tmSA, 0, (m_blk * 2 + (int)rank) * KT + kt, bar);
        tma_load_2d_pair(st + L::A_BYTES + L::B_BYTES + L::SFA_BYTES, &tmSB, 0, (n_blk * 2) * KT + kt, bar);
        tma_load_2d_pair(st + L::A_BYTES + L::B_BYTES + L::SFA_BYTES + 2048, &tmSB, 0, (n_blk * 2 + 1) * KT + kt,
                         bar);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer of the pair (leader only)
    if (rank == 0) {
      constexpr uint32_t idesc = idesc_nvfp4(256, BN);
      uint32_t it = 0, ti = 0;
      bool ok = true;
      for (int t = pair; ok && t < tiles; t += npairs, ++ti) {
        if (ti > 0 && !(ok = __all_sync(0xffffffffu, mbar_wait(acc_empty, (ti - 1) & 1, 114)))) break;
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % L::STAGES;
          const uint32_t ph = (it / L::STAGES) & 1;
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ph, 112)))) break;
          tc_fence_after();
          uint8_t* st = smem + s * L::STAGE_BYTES;
          const uint32_t a_s = smem_u32(st), b_s = smem_u32(st + L::A_BYTES);
          const uint32_t sfa_s = smem_u32(st + L::A_BYTES + L::B_BYTES);
          const uint32_t sfb_s = sfa_s + L::SFA_BYTES;
          const uint32_t sf_t = tmem + 256 + s * L::SF_COLS;
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {
            tmem_cp_pair_32x128b_x4(sf_t + 4 * kb, sdesc_sf_atom(sfa_s + kb * 512));
#pragma unroll
            for (int nb = 0; nb < 2; ++nb)
              tmem_cp_pair_32x128b_x4(sf_t + 16 + 8 * kb + 4 * nb, sdesc_sf_atom(sfb_s + nb * 2048 + kb * 512));
          }
#pragma unroll
          for (int kb = 0; kb < 4; ++kb)
            mma_nvfp4_pair(tmem, sdesc_kmajor_sw128(a_s + kb * 32), sdesc_kmajor_sw128(b_s + kb * 32), idesc,
                           sf_t + 4 * kb, sf_t + 16 + 8 * kb, (kt | kb) != 0);
          tc_commit_pair(&empty[s], 0x3);
        }
        tc_commit_pair(acc_full, 0x3);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs, their own 128 rows)
    const int q = warp & 3;
    const int cofs = ((warp - 2) >> 2) * CW;
    const float alpha = p.a_slot->act * p.g_b;
    const float inv_q = EPI == H3_EPI_ACT_Q ? __fdiv_rn(1.0f, p.q_slot->act) : 0.f;
    const int F = p.act_kind ? (p.N >> 1) : p.N;
    const uint32_t leader_acc_empty = cluster_addr(acc_empty, 0);
    float amax = 0.f;
    uint32_t ti = 0;
    for (int t = pair; t < tiles; t += npairs, ++ti) {
      const int m_blk = t / tiles_n, n0 = (t % tiles_n) * BN;
      const int row = m_blk * 256 + (int)rank * 128 + q * 32 + lane;
      const bool live = row < p.M;
      __nv_bfloat16* xrow;
      const float* gate;
      epi_prefetch<EPI, CW>(p, row, n0 + cofs, xrow, gate);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, ti & 1, 113));
      if (!ok) break;
      tc_fence_after();
      uint32_t hold[CW / 2];
      epi_load<CW>(hold, tmem, q, cofs, n0 + cofs, alpha, p.bias);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_acc_empty);
      if (!live) continue;
      epi_store<EPI, CW>(p, hold, row, n0 + cofs, xrow, gate, inv_q, F, amax);
    }
    if (p.q_slot && (EPI == H3_EPI_ACT_BF16 || EPI == H3_EPI_ACT_Q)) {
      amax = warp_max(amax);
      if (lane == 0) atomic_max_pos(&p.q_slot->amax, amax);
    }
  }
  tc_fence_before();
  cluster_sync();   // every MMA of the pair done, every remote arrival delivered, before TMEM and smem go
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, L::TMEM_COLS);
}

}  // namespace h3
