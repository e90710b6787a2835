/* libh3b200 -- C ABI of the B200 (sm_100a) MiniMax H3 DiT block hot path.
 *
 * Every entry point takes raw device pointers, explicit sizes / strides and a CUDA stream (`stream` is a
 * cudaStream_t passed as void*; NULL = the legacy default stream), launches asynchronously, allocates nothing
 * (scratch comes from the caller) and returns an int status: 0 on success, a negative H3_ERR_* code otherwise, with
 * a message for h3_last_error().  No C++ exception crosses the boundary.  All bf16 tensors are row-major with the
 * given row stride in elements; NVFP4 tensors are e2m1 codes (two a byte, even element in the low nibble) plus one
 * e4m3 scale per 16 elements and one fp32 global scale.
 *
 * Each declaration names the reference interface it replaces (jayleaton/minimax-h3-tensorfold-rtx, file:line).
 */
#ifndef H3B200_H
#define H3B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3B200_VERSION 1

enum {
  H3_OK = 0,
  H3_ERR_ARG = -1,     /* null / misaligned pointer, bad enum value */
  H3_ERR_SHAPE = -2,   /* unsupported size (see each entry point) */
  H3_ERR_CUDA = -3,    /* a CUDA runtime / driver call failed */
  H3_ERR_DEVICE = -4   /* a kernel's bounded wait gave up (h3_device_status holds where) */
};

/* GEMM epilogues (h3_gemm_nvfp4). */
enum {
  H3_EPI_STORE = 0,       /* out = bf16(acc * gA * gB + bias) */
  H3_EPI_GATE_RESID = 1,  /* x = bf16(x + bf16(acc * gA * gB + bias) * gate[idx[row]]): gate_add fused */
  H3_EPI_ACT_BF16 = 2,    /* out = bf16(act(bf16(y))), amax of it into q_slot */
  H3_EPI_ACT_Q = 3,       /* act as above, quantised to NVFP4 under q_slot->act (and amax into q_slot) */
  H3_EPI_STORE_PEERS = 4  /* STORE, each head's columns into the receive buffer of the rank that owns the head */
};

/* Activation-scale state of one linear input (16 bytes, device memory).  amax: max |input| seen this forward
 * (-1 = none); act: the global scale the quantiser uses now; used: the delayed scale in use (0 = none); margin:
 * delayed-scale margin (0 = unset, i.e. 2).  Mirrors Nvfp4Linear.amax_dev / lin.act / used_act / margin,
 * tfvideo/linear.py:113-154. */
typedef struct H3ScaleSlot {
  float amax;
  float act;
  float used;
  float margin;
} H3ScaleSlot;

/* Fused-epilogue parameters of h3_gemm_nvfp4 (fields not used by `kind` are ignored). */
typedef struct H3Epilogue {
  int kind;              /* H3_EPI_* */
  void* out;             /* bf16: STORE / ACT_BF16 output; ACT_Q: optional bf16 copy of the activation (NULL = none) */
  long long ldo;
  void* x;               /* GATE_RESID: bf16 residual [M, N], updated in place */
  long long ldx;
  const float* mod;      /* GATE_RESID: fp32 modulation rows [R, 6, N] */
  const int* idx;        /* GATE_RESID: int32 [M] modulation row of each row */
  int gate_part;         /* 0: gate_msa (chunk 2), 1: gate_mlp (chunk 5) */
  int act_kind;          /* ACT_*: 0 gelu_tanh (F = N), 1 swiglu on 16-column interleaved [gate | up] (F = N / 2) */
  uint8_t* qcodes;       /* ACT_Q: NVFP4 codes [M, F / 2] */
  uint8_t* qsf;          /* ACT_Q: tiled scales (see h3_sf_tiled_bytes) */
  H3ScaleSlot* q_slot;   /* ACT_*: the activation's scale slot */
  /* STORE_PEERS (Ulysses sequence parallelism; no counterpart in the reference, which runs on one GPU): the GEMM's
   * M rows are this rank's M tokens of qkv, N = 3 H 128.  Element (row, part, head, d) is stored to
   * peer[head / Hr] at bf16 element ((rank * M + row) * 3 + part) * Hr * 128 + (head % Hr) * 128 + d, Hr = H / ranks:
   * every rank's [ranks * M, 3, Hr, 128] receive buffer gets all tokens of its heads.  peer[r] is rank r's buffer as
   * mapped in this process (h3_peer_alloc / h3_peer_open), or any base the rows for rank r are to be offset from
   * (e.g. a local staging buffer that h3_peer_push then sends in contiguous blocks). */
  void* peer[8];
  int ranks;             /* 1..8; N % (3 * 128 * ranks) == 0 */
  int rank;
} H3Epilogue;

/* ---------------------------------------------------------------------------------------------- library */
int h3_version(void);
/* Copies the calling thread's last error message (NUL-terminated, truncated to n). Returns its full length. */
int h3_last_error(char* buf, int n);
/* Reads the device status word of the current device (0 = ok; else the code of the wait that gave up) and clears it
 * when reset != 0.  Synchronous. */
int h3_device_status(int* status, int reset);
/* In stream order, *dst = max(*dst, status word of the current device): a collective (max) over this value after a
 * kernel lets every rank learn, on the device and without a host read, that some rank's bounded wait gave up.  No
 * counterpart in the reference (one GPU). */
int h3_status_publish(float* dst, void* stream);
/* Bytes of a tiled NVFP4 scale buffer for `rows` x `cols` elements: ceil(rows / 128) * 128 * cols / 16.  The GEMM
 * reads A and B scales in this layout (512-byte atoms of 128 rows x 4 groups: byte
 * (r % 32) * 16 + (r / 32 % 4) * 4 + g % 4 of atom [r / 128][g / 4]). */
size_t h3_sf_tiled_bytes(int rows, int cols);

/* ---------------------------------------------------------------------------------------------- scales */
/* Start a forward for n slots: delayed = 0 resets every slot (replaces reset_delayed, tfvideo/linear.py:213-216);
 * delayed = 1 turns each slot's amax of the last forward into this forward's act (replaces update_delayed,
 * tfvideo/linear.py:192-210, with no host read); *clipped (device int, nullable) += clipped slots. */
int h3_scales_begin(H3ScaleSlot* slots, int n, int delayed, int* clipped, void* stream);
/* slot->act = max(slot->amax, 1e-6) / 2688: the dynamic per-call scale (tfvideo/linear.py:146-149). */
int h3_scales_dynamic(H3ScaleSlot* slot, void* stream);
/* *out = max(*out, max |x|) over a bf16 [R, K] matrix (replaces linear.absmax, tfvideo/linear.py:41-45). */
int h3_absmax_bf16(const void* x, long long ldx, int R, int K, float* out, void* stream);

/* ---------------------------------------------------------------------------------------------- elementwise */
/* RMSNorm(x) * w * (1 + scale[idx]) + shift[idx] (replaces kernels.norm_mod, tfvideo/kernels.py:15-40), D % 16 == 0
 * and D <= 6144.  Outputs (each optional, at least one): bf16 `out`; NVFP4 `codes` [S, D/2] + `sf` (tiled when
 * sf_tiled, else row-major [S, D/16]) quantised under slot->act; slot->amax accumulates max |y| when slot given. */
int h3_norm_mod(const void* x, int ldx, const float* w, const float* mod, const int* idx, int S, int D, int part,
                float eps, void* out, int ldo, uint8_t* codes, uint8_t* sf, int sf_tiled, H3ScaleSlot* slot,
                void* stream);
/* bf16 [R, K] -> NVFP4 under global scale *g_dev (or g when g_dev is NULL) (replaces TensorFold quant4 and the
 * activation quantiser of prompt(A4, ...), tfvideo/linear.py:30-38,151).  Element (r, c) is read at
 * x + (c / cblk) * blk_stride + r * ldx + c % cblk (cblk = K for a plain matrix).  amax (nullable) += max |x|. */
int h3_nvfp4_quant(const void* x, long long ldx, int cblk, long long blk_stride, int R, int K, const float* g_dev,
                   float g, uint8_t* codes, uint8_t* sf, int sf_tiled, float* amax, void* stream);
/* x += y * gate[idx] in place (replaces kernels.gate_add, tfvideo/kernels.py:43-63), D % 8 == 0. */
int h3_gate_add(void* x, int ldx, const void* y, int ldy, const float* mod, const int* idx, int S, int D, int part,
                void* stream);
/* act_kind 0: gelu_tanh(u) (u [M, F]); 1: silu(gate) * up (u = [gate | up] [M, 2F]) (replaces kernels.swiglu,
 * tfvideo/kernels.py:66-84); bf16 out [M, F]; amax (nullable) += max |out|.  F % 8 == 0. */
int h3_act(const void* u, int ldu, void* out, int ldo, int M, int F, int act_kind, float* amax, void* stream);
/* mod[m, j] = ada_b[j] + t_emb[m] . ada_w[j] (fp32 [M, J]) (replaces MiniMaxH3Engine.modulation,
 * tfvideo/minimax_h3.py:265-269). */
int h3_modulation(const float* t_emb, int M, int t_dim, const float* ada_w, const float* ada_b, int J, float* mod,
                  void* stream);

/* ---------------------------------------------------------------------------------------------- peer memory */
/* Device buffers other processes on the node map (CUDA IPC), the receive buffers of the fused Ulysses exchanges.
 * No counterpart in the reference (one GPU).  h3_peer_alloc allocates `bytes` on the current device and writes its
 * 64-byte IPC handle to `handle`; another process passes that handle to h3_peer_open to map the buffer (peer access
 * enabled on demand).  Close mappings before the owner frees the buffer. */
int h3_peer_alloc(size_t bytes, void** ptr, void* handle);
int h3_peer_open(const void* handle, void** ptr);
int h3_peer_close(void* ptr);
int h3_peer_free(void* ptr);
/* One contiguous device-to-device copy of h3_peer_push: src and dst 16-byte aligned, bytes a multiple of 16. */
typedef struct H3PeerCopy {
  const void* src;
  void* dst;
  size_t bytes;
} H3PeerCopy;
/* Up to 8 copies in one kernel, typically into other ranks' peer buffers: every warp stores 512 contiguous bytes at a
 * time, so writes to another GPU cross NVLink in full packets (row-scattered 16-byte stores do not).  The grid is
 * about one 128-thread block per SM over all copies, small enough to sit beside a persistent h3_gemm_nvfp4 CTA, so a
 * push on another stream runs while the GEMM does.  Like any kernel's, its writes are visible to work ordered after
 * its completion (for another rank: after a barrier). */
int h3_peer_push(const H3PeerCopy* copies, int n, void* stream);
/* The same copies (any number) as cudaMemcpyAsync device-to-device calls on `stream`, one per copy: the copy engines
 * move the data, so it overlaps kernels that hold every SM (a persistent GEMM). */
int h3_peer_copy(const H3PeerCopy* copies, int n, void* stream);

/* ---------------------------------------------------------------------------------------------- GEMM */
/* NVFP4 W4A4 GEMM y = A x B^T (replaces Nvfp4Linear.__call__ -> TensorFold prompt(A4, x, lin),
 * tfvideo/linear.py:141-151): A codes [M, K/2] and tiled scales (h3_sf_tiled_bytes(M, K)) with global scale
 * a_slot->act; B codes [N, K/2], tiled scales, global scale g_b; bias fp32 [N] or NULL.  K % 256 == 0, N % 128 == 0;
 * codes 16-byte aligned.  The epilogue `epi` fuses the consumer of y (see H3_EPI_*). */
int h3_gemm_nvfp4(const uint8_t* a_codes, const uint8_t* a_sf, const H3ScaleSlot* a_slot, const uint8_t* b_codes,
                  const uint8_t* b_sf, float g_b, const float* bias, int M, int N, int K, const H3Epilogue* epi,
                  void* stream);

/* ---------------------------------------------------------------------------------------------- attention */
/* Per-head RMSNorm (weights qw, kw [128]) + split-half RoPE over the first `rot` dims, in place on q and k rows
 * (element (s, h, d) at q + s * ld + h * 128 + d) (replaces comfy_kitchen.rms_rope_split_half_, called at
 * tfvideo/minimax_h3.py:296-298).  rope: fp32 [S, rot/2, 2, 2] rotation matrices; rot % 8 == 0, rot <= 128. */
int h3_qknorm_rope(void* q, void* k, long long ld, int S, int H, int rot, const float* qw, const float* kw,
                   const float* rope, float eps, void* stream);
/* Scratch bytes h3_attn_fp8 needs for S tokens and H heads. */
size_t h3_attn_workspace_bytes(int S, int H);
/* Non-causal FP8 attention softmax(q k^T / sqrt(128)) v over H heads of head_dim 128 (replaces the attention
 * backends of tfvideo/attention.py:44-54 and fp4attn.attention(qk="fp8", pv="fp8"), tfvideo/fp4attn.py:245-290).
 * Element (t, h, d) of q / k / v at base + t * ld + h * hstride + d (bf16); out (t, h, d) at out + t * ldo + h * 128
 * + d (bf16).  workspace: h3_attn_workspace_bytes(S, H) bytes, 1024-byte aligned.  S <= 262,144 and H <= 65,535
 * (H3_ERR_SHAPE beyond). */
int h3_attn_fp8(const void* q, const void* k, const void* v, long long ld, long long hstride, int S, int H, void* out,
                long long ldo, void* workspace, size_t workspace_bytes, void* stream);

/* h3_attn_fp8 under a block-sparse mask of 128 x 128 tiles shared by all heads: query tile qt (tokens 128 qt ..
 * 128 qt + 127) attends only to the KV tiles kv_idx[kv_ptr[qt] .. kv_ptr[qt + 1]) (device int32; kv_ptr has
 * ceil(S / 128) + 1 entries; each list free of duplicates, any order, entries in [0, ceil(S / 128)); an out-of-range
 * entry is skipped and recorded in the device status word).  The softmax runs over the kept keys only; a query tile
 * with an empty list gets zero rows.  This is the "optional block-sparse mask" of the attention path; the reference
 * takes its sparse attention from ComfyUI's BlockSparseAttention node (tfvideo/minimax_h3.py:285-291 hands the block
 * to it), which has no in-repository kernel.  Same workspace as h3_attn_fp8. */
int h3_attn_fp8_sparse(const void* q, const void* k, const void* v, long long ld, long long hstride, int S, int H,
                       const int* kv_ptr, const int* kv_idx, void* out, long long ldo, void* workspace,
                       size_t workspace_bytes, void* stream);

/* h3_attn_fp8 (kv_ptr NULL) or h3_attn_fp8_sparse whose output rows go straight to the ranks that own the tokens
 * (Ulysses sequence parallelism; no counterpart in the reference, which runs on one GPU).  q, k, v hold all S tokens
 * of this rank's H heads; the token t's row of head h goes to peer[t / n] (n = S / ranks) at bf16 element
 * ((rank * n + t % n) * ldo + h * 128 + d): every rank's [ranks, n, ldo] receive buffer gets its n tokens, column
 * block r from rank r's heads.  peer: host array of `ranks` (1..8) buffers as mapped in this process
 * (h3_peer_alloc / h3_peer_open), or any base the rows for rank r are to be offset from (e.g. a local staging buffer
 * that h3_peer_push then sends in contiguous blocks); S % ranks == 0. */
int h3_attn_fp8_peers(const void* q, const void* k, const void* v, long long ld, long long hstride, int S, int H,
                      const int* kv_ptr, const int* kv_idx, void* const* peer, int ranks, int rank, long long ldo,
                      void* workspace, size_t workspace_bytes, void* stream);

/* The same attention as h3_attn_fp8 for callers that cannot allocate device memory -- for example code running
 * inside a host framework that owns every device allocation (ComfyUI records and replays a block's allocations under
 * its dynamic-VRAM mode), or a plugin handed only input and output buffers.  Its scratch is a fixed 64 MiB device
 * array inside this library, held by every GPU that loads the library until the process exits; problems whose
 * h3_attn_workspace_bytes(S, H) exceed 64 MiB - 1 KiB (about S * H <= 170,000, e.g. S = 4096 at H = 40) are
 * rejected with H3_ERR_SHAPE.  The first call on a device looks up the array's device address (make it before any
 * stream capture); the address is kept per CUDA context, so a call made in another context on that device, or after
 * a device reset, looks it up again for that context.  All calls share the array, so calls that overlap on the GPU
 * (other streams, other threads) race; nothing in it needs to start at zero.  It allocates nothing.  This entry point
 * has no counterpart in the reference. */
int h3_attn_fp8_noalloc(const void* q, const void* k, const void* v, long long ld, long long hstride, int S, int H,
                        void* out, long long ldo, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* H3B200_H */
