/*
 * kshipra_b200 -- C ABI of the B200 (sm_100a) quantized forward path.
 *
 * Every entry point takes raw device pointers, int64 sizes and a CUDA stream
 * (passed as void*, a cudaStream_t), launches asynchronously on that stream
 * and returns an int status (KSH_OK = 0, negative on a host-side argument
 * error or a failed launch).  Nothing here allocates: the caller owns every
 * buffer, including the workspaces whose sizes the *_workspace_size helpers
 * report.  Data-dependent errors found on the device (bad block id, slot,
 * position, token id, non-finite weight) are OR-ed into a caller-owned int32
 * status word as KSH_FLAG_* bits; kernels never trap.
 *
 * Workspaces need no initialisation: the entry points that keep completion
 * counters in a workspace (ksh_paged_attention, ksh_lm_head_argmax) clear
 * them on the caller's stream before their kernels run, so a buffer fresh
 * from cudaMalloc (or torch.empty) is a valid workspace.
 *
 * Functions are stateless and may be called from any host thread; calls on
 * one stream are ordered, calls on different streams that share a workspace
 * race.
 *
 * Each declaration names the reference interface it replaces
 * (Hedau0404/Kshipra, path:line).
 */
#ifndef KSHIPRA_B200_H
#define KSHIPRA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (return values) ---- */
#define KSH_OK               0
#define KSH_ERR_SHAPE       -1   /* bad size / shape argument */
#define KSH_ERR_ALIGN       -2   /* pointer not aligned as required */
#define KSH_ERR_CUDA        -3   /* launch failed; see ksh_last_cuda_error() */
#define KSH_ERR_UNSUPPORTED -4   /* shape outside what the kernels handle */
#define KSH_ERR_WORKSPACE   -5   /* workspace missing or too small */
#define KSH_ERR_TOO_LARGE   -6   /* size beyond a fixed scratch array's capacity */

/* ---- device status-word bits ---- */
#define KSH_FLAG_NONFINITE     1   /* weight holds NaN/Inf (QuantizationError) */
#define KSH_FLAG_BAD_BLOCK     2   /* block-table entry outside [0, num_blocks) */
#define KSH_FLAG_BAD_SLOT      4   /* slot outside the pool */
#define KSH_FLAG_BAD_POSITION  8   /* position outside the RoPE table */
#define KSH_FLAG_BAD_TOKEN    16   /* token id outside [0, vocab) */
#define KSH_FLAG_BAD_LENGTH   32   /* sequence longer than its block table */
#define KSH_FLAG_TIMEOUT      64   /* a bounded device wait gave up */

int ksh_abi_version(void);
const char* ksh_status_string(int status);
/* cudaError_t recorded by the last call that returned KSH_ERR_CUDA. */
int ksh_last_cuda_error(void);
/* Enable (1) / disable (0) programmatic dependent launch; returns previous. */
int ksh_set_pdl(int enabled);
/* Enable (1) / disable (0) the register-resident decode GEMV for small
 * matrices (disabled: the streaming GEMV serves all M <= 16); returns previous. */
int ksh_set_gemv_resident(int enabled);
/* Tensor-core decode path for quantized linears with m <= 16 (swap-AB tcgen05
 * kernels): 0 off, 1 auto (by scheme, m and matrix size), 2 every eligible
 * shape, 3 as 2 with INT8 through the fp16-operand kernel (tests).  Returns the
 * previous mode.  A tuning switch with no counterpart in the reference;
 * results agree with the CUDA-core path within fp32 rounding. */
int ksh_set_gemv_tc(int mode);
/* One-row INT4 linears through the dp4a kernel (exact int32 products of the
 * nibbles with three 8-bit digits of x): 1 on (default), 0 off (the GEMV /
 * tensor-core paths take them).  Returns the previous setting.  A tuning
 * switch with no counterpart in the reference. */
int ksh_set_gemv_dp4a(int enabled);
/* Quantized linears with 17..64 rows through the swap-AB tensor-core kernel
 * (weight rows on the MMA's 128 lanes, token rows on its N side): 1 on
 * (default), 0 off (the prefill GEMM takes them).  Returns the previous
 * setting.  A tuning switch with no counterpart in the reference; results
 * agree with the prefill GEMM within fp32 rounding. */
int ksh_set_gemm_mid(int enabled);
/* Rows of x from which the prefill GEMM first widens the whole quantized
 * weight to fp16 in the workspace (one pass, exact) and then streams fp16
 * tiles by TMA straight into the MMA (default 512; 0 never;
 * KSH_GEMM_PREDEQ_MIN in the environment sets it at load).  Below it each
 * output tile widens its own weight tiles.  ksh_linear_workspace_size counts
 * the fp16 copy for such m.  Returns the previous setting.  A tuning switch
 * with no counterpart in the reference; results are identical either way. */
int64_t ksh_set_gemm_predeq(int64_t min_rows);
/* Key split of ksh_decode_attention: the number of CTAs (one thread-block
 * cluster) that share a (sequence, kv head), 1..8; 0 or out of range restores
 * the per-launch choice (waves of resident CTAs x keys per CTA).  Returns the
 * previous setting.  A tuning switch with no counterpart in the reference;
 * results agree across splits within fp32 rounding. */
int ksh_set_decode_split(int clusters);
/* The same for ksh_decode_attention_ws: CTAs per (sequence, kv head) of the
 * cluster-free key split, 1..8 (1 runs the unsplit kernel); 0 restores the
 * per-launch choice.  KSH_DECODE_GSPLIT=1..8 in the environment sets it at
 * load.  Returns the previous setting.  No counterpart in the reference. */
int ksh_set_decode_gsplit(int splits);
/* Kernels this library has launched since it was loaded, counting those
 * recorded into a CUDA graph under capture (a replay of that graph launches
 * them again without counting). */
uint64_t ksh_kernel_launches(void);

/* ------------------------------------------------------------------------
 * Weight packing.  w: fp32 [n, k] row-major.
 * ---------------------------------------------------------------------- */

/* Replaces quantize_int8_per_channel, engine/quantization.py:196-223.
 * payload int8 [n, k]; scales fp16 bits [n]. */
int ksh_pack_int8(const float* w, int64_t n, int64_t k, int8_t* payload,
                  uint16_t* scales, int32_t* flags, void* stream);

/* Replaces quantize_int4_per_group, engine/quantization.py:238-318.
 * group_size even and > 0; k_padded = ceil(k / g) * g;
 * payload uint8 [n, k_padded / 2] (low nibble = even k);
 * scales fp16 bits [n, k_padded / g]. */
int ksh_pack_int4(const float* w, int64_t n, int64_t k, int64_t group_size,
                  uint8_t* payload, uint16_t* scales, int32_t* flags, void* stream);

/* ------------------------------------------------------------------------
 * Linear layers (replace QuantizedLinear.forward, engine/quantization.py:
 * 394-396, and nn.Linear for unquantized weights):
 *   y[m, j] = sum_k x'[m, k] * W[j, k] + bias[j] + residual[m, j]
 * x fp32 [m, k]; bias [n] or NULL; residual [m, n] or NULL (may alias y).
 * norm_w [k] or NULL: when set, x' = RMSNorm(x) with that weight and
 * norm_eps (LlamaRMSNorm, engine/model.py:113,146), fused into the load of
 * x; when NULL, x' = x.
 * M <= 16 runs the decode GEMV; larger M the tensor-core GEMM, which needs
 * the workspace reported by ksh_linear_workspace_size (else NULL/0).
 * ---------------------------------------------------------------------- */
int64_t ksh_linear_workspace_size(int64_t m, int64_t k, int64_t n);

int ksh_qlinear_w8(const float* x, int64_t m, int64_t k,
                   const float* norm_w, float norm_eps, const int8_t* payload,
                   const uint16_t* scales, const float* bias, const float* residual,
                   float* y, int64_t n, void* workspace, int64_t workspace_bytes,
                   void* stream);

int ksh_qlinear_w4(const float* x, int64_t m, int64_t k,
                   const float* norm_w, float norm_eps, const uint8_t* payload,
                   const uint16_t* scales, int64_t group_size, int64_t k_padded,
                   const float* bias, const float* residual, float* y, int64_t n,
                   void* workspace, int64_t workspace_bytes, void* stream);

int ksh_linear_f32(const float* x, int64_t m, int64_t k,
                   const float* norm_w, float norm_eps, const float* w,
                   const float* bias, const float* residual, float* y, int64_t n,
                   void* workspace, int64_t workspace_bytes, void* stream);

/* Gate/up projection fused with SwiGLU (replaces LlamaMLP's
 * act(gate_proj(x)) * up_proj(x), called at engine/model.py:147):
 * the weight holds 2*inter rows, gate rows [0, inter) then up rows
 * [inter, 2*inter); h[m, j] = silu(g[m, j]) * u[m, j]. */
int ksh_qlinear_swiglu_w8(const float* x, int64_t m, int64_t k,
                   const float* norm_w, float norm_eps, const int8_t* payload,
                          const uint16_t* scales, float* h, int64_t inter,
                          void* workspace, int64_t workspace_bytes, void* stream);
int ksh_qlinear_swiglu_w4(const float* x, int64_t m, int64_t k,
                   const float* norm_w, float norm_eps, const uint8_t* payload,
                          const uint16_t* scales, int64_t group_size, int64_t k_padded,
                          float* h, int64_t inter, void* workspace,
                          int64_t workspace_bytes, void* stream);
int ksh_linear_swiglu_f32(const float* x, int64_t m, int64_t k,
                   const float* norm_w, float norm_eps, const float* w,
                          float* h, int64_t inter, void* workspace,
                          int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Embedding + RMSNorm (HF Embedding / LlamaRMSNorm, engine/model.py:107,113,
 * 146,150).  rmsnorm: y = w * (x * rsqrt(mean(x^2) + eps)), fp32.
 * ---------------------------------------------------------------------- */
int ksh_embedding(const int64_t* ids, int64_t m, const float* table, int64_t vocab,
                  int64_t hidden, float* out, int32_t* flags, void* stream);
int ksh_rmsnorm(const float* x, const float* w, float* y, int64_t m, int64_t hidden,
                float eps, void* stream);

/* ------------------------------------------------------------------------
 * RoPE at absolute positions + K/V scatter into the block pool
 * (replaces _apply_rope + the per-token pool write, engine/model.py:108,121,
 * 123-129).  qkv fp32 [m, (hq + 2*hkv) * d] (q heads, then k, then v);
 * rope_cos / rope_sin fp32 [max_pos, d/2] (cos/sin of position * inv_freq);
 * q_out fp32 [m, hq, d]; pool fp32 [num_blocks, num_layers, 2, hkv,
 * block_size, d]; slot = block_id * block_size + offset.
 * ---------------------------------------------------------------------- */
int ksh_rope_kv_write(const float* qkv, int64_t m, int64_t hq, int64_t hkv, int64_t d,
                      const int64_t* positions, const int64_t* slot_mapping,
                      const float* rope_cos, const float* rope_sin, int64_t max_pos,
                      float* q_out, float* pool, int64_t num_blocks, int64_t num_layers,
                      int64_t layer, int64_t block_size, int32_t* flags, void* stream);

/* ------------------------------------------------------------------------
 * Paged online-softmax attention over the block pool (replaces
 * chunked_attention, engine/chunked_prefill.py:93-140), batched over
 * sequences (varlen).  Sequence s owns query rows [q_start[s], q_start[s+1])
 * of q [T, hq, d], at absolute positions prefix_lens[s] + i; it attends to
 * keys 0 .. prefix_lens[s] + len - 1 stored through
 * block_tables[s * max_blocks + j] with a causal mask.  GQA: query head h
 * reads kv head h / (hq / hkv).  q_start / prefix_lens live on the device
 * (they may change between graph replays); max_q_len and max_total_len are
 * host-side upper bounds used to size the grid.
 * ---------------------------------------------------------------------- */
int64_t ksh_paged_attention_workspace_size(int64_t num_seqs, int64_t hq, int64_t hkv,
                                           int64_t d, int64_t max_q_len,
                                           int64_t max_total_len);
int ksh_paged_attention(const float* q, int64_t hq, int64_t d, const float* pool,
                        int64_t num_blocks, int64_t num_layers, int64_t layer,
                        int64_t hkv, int64_t block_size, const int32_t* block_tables,
                        int64_t max_blocks, const int32_t* q_start,
                        const int32_t* prefix_lens, int64_t num_seqs, int64_t max_q_len,
                        int64_t max_total_len, float* out, void* workspace,
                        int64_t workspace_bytes, int32_t* flags, void* stream);

/* ------------------------------------------------------------------------
 * Decode step fused: RoPE of the new token's q / k at positions[b], the K/V
 * write into the pool at slot_mapping[b], and paged attention of the token
 * over keys 0 .. positions[b] (replaces _apply_rope + the pool write,
 * engine/model.py:108,121-129, and chunked_attention with chunk_len = 1,
 * engine/chunked_prefill.py:93-140).  qkv [batch, (hq + 2*hkv) * d] as for
 * ksh_rope_kv_write; out [batch, hq, d].  Needs block_size % 16 == 0 and
 * d in {64, 128}; max_total_len bounds positions[b] + 1 (grid sizing).
 * ---------------------------------------------------------------------- */
int ksh_decode_attention(const float* qkv, int64_t batch, int64_t hq, int64_t hkv, int64_t d,
                         const int64_t* positions, const int64_t* slot_mapping,
                         const float* rope_cos, const float* rope_sin, int64_t max_pos,
                         float* pool, int64_t num_blocks, int64_t num_layers, int64_t layer,
                         int64_t block_size, const int32_t* block_tables, int64_t max_blocks,
                         int64_t max_total_len, float* out, int32_t* flags, void* stream);

/* The same fused decode step with a workspace for key-split partial
 * states: the keys of each (sequence, kv head) are split over independent
 * CTAs (1..8, chosen per launch so that the CTAs fill the SMs' resident
 * slots) whose online-softmax states the last one to finish merges in split
 * order; without the workspace the split is a thread-block cluster.  The
 * workspace, of ksh_decode_attention_workspace_size(batch, hq, hkv, d) bytes
 * and 256-byte aligned, must be zero before its first use; every launch
 * leaves its counters at zero again, so a CUDA graph can replay the call
 * without a memset in between. */
int64_t ksh_decode_attention_workspace_size(int64_t batch, int64_t hq, int64_t hkv, int64_t d);
int ksh_decode_attention_ws(const float* qkv, int64_t batch, int64_t hq, int64_t hkv, int64_t d,
                            const int64_t* positions, const int64_t* slot_mapping,
                            const float* rope_cos, const float* rope_sin, int64_t max_pos,
                            float* pool, int64_t num_blocks, int64_t num_layers, int64_t layer,
                            int64_t block_size, const int32_t* block_tables, int64_t max_blocks,
                            int64_t max_total_len, float* out, void* workspace,
                            int64_t workspace_bytes, int32_t* flags, void* stream);

/* ------------------------------------------------------------------------
 * lm_head (fp32, never quantized; engine/model.py:151) fused with the greedy
 * argmax of generate (model.py:187, 200; first index of the maximum, as
 * torch.argmax).  logits [m, vocab] may be NULL (argmax only); norm_w as for
 * the linear layers (the final model.norm, model.py:150).
 * ---------------------------------------------------------------------- */
int64_t ksh_lm_head_workspace_size(int64_t m, int64_t vocab);
int ksh_lm_head_argmax(const float* x, int64_t m, int64_t hidden, const float* norm_w,
                       float norm_eps, const float* w,
                       int64_t vocab, float* logits, int64_t* tokens, void* workspace,
                       int64_t workspace_bytes, void* stream);
/* The same lm_head + greedy argmax (fused GEMV path only) for callers that
 * cannot allocate device memory: an FFI binding handed only device pointers
 * by a host runtime whose allocator it cannot reach, or a latency-critical
 * loop that must not call cudaMalloc (it can synchronize the device).  No
 * counterpart in the reference.
 * Scratch is a fixed 256 KiB device array per GPU (its size:
 * ksh_lm_head_argmax_noalloc_max_bytes()); m <= 16 and vocabularies whose
 * partials fit it, else KSH_ERR_TOO_LARGE.  The first call on a device looks
 * up the array's address (make it before any stream capture).  All calls
 * share the array: calls that overlap on the GPU race.  Allocates nothing. */
int64_t ksh_lm_head_argmax_noalloc_max_bytes(void);
int ksh_lm_head_argmax_noalloc(const float* x, int64_t m, int64_t hidden, const float* norm_w,
                               float norm_eps, const float* w, int64_t vocab, float* logits,
                               int64_t* tokens, void* stream);
/* The same lm_head (+ argmax) on tcgen05 tensor cores for many rows (the
 * decode step of a large batch, the L-row logits of a prefill forward).
 * The fp32 weight is split once by ksh_lm_head_split_weight into fp16
 * w_hi, w_lo [vocab, hidden] and w_inv [vocab] (per row a power-of-two
 * scale 2^s with max|w| * 2^s in [2^14, 2^15): w * 2^s = hi + lo, w_inv =
 * 2^-s; non-finite weights raise KSH_FLAG_NONFINITE in *flags).  Each call
 * splits x the same way (RMSNorm folded in) and runs W_hi x (x_hi + x_lo) +
 * W_lo x x_hi with fp32 accumulation, so only the lo x lo term (about 2^-22
 * of each product) is dropped.  Any m (64 rows per launch, one pass over the
 * weight each); hidden % 8 == 0; 16-byte aligned w_hi / w_lo; workspace of
 * ksh_lm_head_tc_workspace_size(m, hidden, vocab) bytes, 256-byte aligned. */
int64_t ksh_lm_head_tc_workspace_size(int64_t m, int64_t hidden, int64_t vocab);
int ksh_lm_head_split_weight(const float* w, int64_t vocab, int64_t hidden, void* w_hi,
                             void* w_lo, float* w_inv, int32_t* flags, void* stream);
int ksh_lm_head_argmax_tc(const float* x, int64_t m, int64_t hidden, const float* norm_w,
                          float norm_eps, const void* w_hi, const void* w_lo, const float* w_inv,
                          int64_t vocab, float* logits, int64_t* tokens, void* workspace,
                          int64_t workspace_bytes, void* stream);
/* Row-wise argmax of materialised logits [m, vocab]. */
int ksh_argmax_rows(const float* logits, int64_t m, int64_t vocab, int64_t* out,
                    void* stream);

/* ------------------------------------------------------------------------
 * Greedy decode bookkeeping on the device, so a decode step can be replayed
 * from a CUDA graph without a host round trip (replaces the host side of
 * generate's loop, engine/model.py:194-203).  For each sequence b:
 *   ids[b] = next[b]; history[b * hist_stride + step[0]] = next[b];
 *   positions[b] += 1; prefix_lens[b] = positions[b];
 *   slots[b] = block_tables[b * max_blocks + pos / B] * B + pos % B
 * and step[0] += 1 (once).
 * ---------------------------------------------------------------------- */
int ksh_decode_advance(const int64_t* next, int64_t batch, int64_t* ids,
                       int64_t* positions, int32_t* prefix_lens, int64_t* slots,
                       const int32_t* block_tables, int64_t max_blocks,
                       int64_t block_size, int64_t* history, int64_t hist_stride,
                       int64_t* step, int32_t* flags, void* stream);

/* ------------------------------------------------------------------------
 * Sum all-reduce of the tensor-parallel partial sums over peer memory (one
 * process per GPU; the reference is single-process and has none: this
 * replaces the collective after the row-parallel o_proj / down_proj of this
 * build's sharded KshipraModel.forward, engine/model.py:111-148).
 * peer_buffers: device array of `world` pointers, every rank's buffer of
 * ksh_peer_allreduce_buffer_floats(n_max, world) floats mapped into this
 * process (symmetric memory), zeroed before the first call.  A call sums the
 * n floats (n % 4 == 0, n <= n_max) each rank left at float offset
 * parity * n_max of its buffer into out (reduce-scatter + all-gather over
 * plain peer loads; each slice summed once in rank order, so every rank
 * gets the same bits).  Consecutive calls must alternate parity 0 / 1 and
 * come in the same order on every rank.  epochs: ksh_peer_allreduce_epoch_words()
 * zeroed words of device memory per rank.  Waits for peers are bounded
 * (KSH_FLAG_TIMEOUT in *flags).
 * ---------------------------------------------------------------------- */
int64_t ksh_peer_allreduce_buffer_floats(int64_t n_max, int world);
int64_t ksh_peer_allreduce_epoch_words(void);
int ksh_peer_allreduce_f32(const uint64_t* peer_buffers, int rank, int world, int64_t n,
                           int64_t n_max, int parity, float* out, uint32_t* epochs,
                           int32_t* flags, void* stream);

/* ------------------------------------------------------------------------
 * Failure-path check of the device waits (no counterpart in the reference;
 * it stands in for the reference's timeout-and-report handling of a stuck
 * worker, benchmarks/run_benchmarks.py:234-267, at the device level).  One
 * CTA waits, with the same bounded primitives the pipelined kernels use, on
 * an mbarrier phase and on the device word *wait_flag; unless `arrive` is
 * set nothing completes either, so each wait gives up after `polls` attempts
 * (1 .. 2^24), KSH_FLAG_TIMEOUT is OR-ed into *flags and *where (optional)
 * gets bit 0 for the mbarrier, bit 1 for the flag.  The kernel then returns,
 * leaving the context usable.
 * ---------------------------------------------------------------------- */
int ksh_check_bounded_wait(int64_t polls, int arrive, const int32_t* wait_flag,
                           int32_t* flags, int32_t* where, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KSHIPRA_B200_H */
