/*
 * klgemm.h -- C-ABI of the fused KL-GEMM distillation loss for B200 (sm_100a).
 *
 * Replaces the reference's loss path, which has no native FFI of its own:
 * the Python entry point is compute_kl_loss (train.py:142-195), its compiled
 * chunk body _kl_chunk_body (train.py:198-210), and the teacher-probability
 * precompute it consumes (train.py:549-567).  The binding a Python caller
 * uses (ctypes) is orthrus_training_test_b200/_lib.py, which the drop-in
 * compute_kl_loss shim (orthrus_training_test_b200/loss.py) calls.
 *
 * Math (natural log, z = h W^T / T, W = lm_head weight [V, H]):
 *   KL_i  = sum_v p_v (z_t - z_s) - lse(z_t) + lse(z_s),  p = softmax(z_t)
 *   loss  = sum_i valid_i KL_i / count,   count = sum_i valid_i
 *   dZ_s  = g * valid_i / count * (softmax(z_s) - p) / T
 *   dH_s  = dZ_s W,   dW = dZ_s^T h_s   (teacher detached, as in train.py:183)
 *
 * Conventions
 *   - Inputs h_s, h_t [N, H] and W [V, H] are bf16, row-major, 16-byte aligned,
 *     H a multiple of 8 and at least 64.  (fp32 callers use the *_f32 entry points, which keep fp32
 *     fidelity, or round with klg_cast_f32_bf16.)
 *   - mask [N] is uint8 (nonzero = row carries loss), the reference's
 *     target != pad_token_id (train.py:163-164).
 *   - Every pointer is device memory owned by the caller; the library holds no
 *     device allocation across calls.  `stream` is a cudaStream_t; work is only
 *     enqueued on it (no host synchronisation).
 *   - Return value: KLG_OK or a KLG_ERR_* code; klg_last_error gives the text
 *     (per host thread).  Device-side pipeline timeouts are reported through
 *     klg_device_status.
 */
#ifndef KLGEMM_H_
#define KLGEMM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KLG_VERSION 100

#define KLG_OK 0
#define KLG_ERR_ARG 1        /* bad shape, null pointer, inconsistent sizes      */
#define KLG_ERR_ALIGN 2      /* pointer / stride alignment                        */
#define KLG_ERR_CUDA 3       /* CUDA runtime or driver error at launch            */
#define KLG_ERR_WORKSPACE 4  /* workspace missing or too small                    */

/* Library version (KLG_VERSION). */
int klg_version(void);

/* Copies the calling thread's last error message into buf. */
int klg_last_error(char* buf, int len);

/* Reads (and optionally clears) the device status word: 0 = no device-side
 * error; otherwise bits of the pipeline waits that ran out of their time
 * bound (the kernel then ended early).  Synchronises the device. */
int klg_device_status(int* status, int reset);

/* Device status bits. */
#define KLG_STATUS_TIMEOUT_PRODUCER 0x1   /* a TMA producer waited out its bound on a free stage   */
#define KLG_STATUS_TIMEOUT_MMA 0x2        /* the MMA issuer waited out its bound on operands/TMEM  */
#define KLG_STATUS_TIMEOUT_EPILOGUE 0x4   /* an epilogue warp waited out its bound on a tile       */
#define KLG_STATUS_TIMEOUT_DRAIN 0x8      /* a final drain of copies / MMAs waited out its bound   */
#define KLG_STATUS_TIMEOUT_PEER 0x10      /* a cross-rank exchange waited out its bound on a peer  */
#define KLG_STATUS_SELFTEST 0x100         /* set by klg_selftest_wait_timeout                      */

/* Test hook (no counterpart in the reference): launches one block that waits on an
 * mbarrier nothing will complete, through the same bounded wait every pipeline uses.
 * After the bound (~1 s) the wait gives up, sets KLG_STATUS_SELFTEST and the block
 * exits normally, so the context stays usable.  Exercises the timeout path without
 * faulting the GPU. */
int klg_selftest_wait_timeout(void* stream);

/* Number of kernels this library has launched in this process. */
long long klg_launch_count(void);

/* ---------------------------------------------------------------- forward
 * Replaces: the teacher lm_head + softmax + entropy precompute
 * (train.py:549-567 and train.py:188-191), the student lm_head + soft-target
 * cross_entropy + masked sum (train.py:198-210) and the final division
 * (train.py:195).  No [N, V] tensor is formed. */

/* Number of vocab-range partial records klg_fwd_stats writes per row on the
 * current device. */
int klg_num_partials(int64_t n_rows, int64_t vocab, int* n_part);

/* Pass 1: per row, online softmax statistics of both views over W's rows,
 * written as n_part records partials[n_part][5][n_rows] =
 * (m_s, S_s, m_t, S_t, A) in the log2 domain (u = z log2(e)):
 * S = sum 2^(u - m), A = sum_v 2^(u_t - m_t) (u_t - u_s). */
int klg_fwd_stats(const void* h_s, const void* h_t, const void* w, int64_t n_rows, int64_t hidden,
                  int64_t vocab, float inv_temp, float* partials, int n_part, void* stream);

/* Online-softmax merge of partial records [n_part][5][n_rows] -> stats [5][n_rows].
 * Also merges records gathered from ranks holding different vocab shards. */
int klg_merge_stats(const float* partials, int n_part, int64_t n_rows, float* stats, void* stream);

/* count = sum(mask) as a float device scalar (train.py:165). */
int klg_count_valid(const uint8_t* mask, int64_t n_rows, float* count, void* stream);

/* loss = sum(mask * KL) / count (0 when count == 0, train.py:166-167 and 195);
 * lse [2][n_rows] = log2-domain log-sum-exp of (student, teacher) for the
 * backward; row_kl [n_rows] (nats, may be NULL). */
int klg_finalize(const float* stats, const uint8_t* mask, int64_t n_rows, const float* count, float* loss,
                 float* lse, float* row_kl, void* stream);

/* Bytes of forward workspace klg_fwd needs. */
int64_t klg_fwd_workspace_bytes(int64_t n_rows, int64_t vocab);

/* Whole forward on one device: [count] -> stats -> merge -> finalize.
 * count_given = 0: count is computed from mask into *count;
 * count_given = 1: *count already holds the (e.g. all-reduced) normaliser. */
int klg_fwd(const void* h_s, const void* h_t, const void* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
            int64_t vocab, float inv_temp, int count_given, float* count, float* loss, float* lse, float* row_kl,
            void* workspace, int64_t workspace_bytes, void* stream);

/* Allocation-free variant of klg_fwd (no counterpart in the reference), for
 * callers that cannot allocate device memory: e.g. a runtime whose device
 * memory is all reserved up front by its own allocator, or a latency-critical
 * loop where cudaMalloc's implicit device-wide synchronisation is not allowed.
 * Same arguments and results as klg_fwd minus the workspace: its scratch is a
 * fixed 16 MiB array inside the library (klg_fwd_noalloc_max_floats() floats)
 * that each GPU loading the library holds until exit; problems needing more,
 * (n_part + 1) * 5 * n_rows floats, are rejected with KLG_ERR_WORKSPACE.  The
 * first call on a device looks up the array's address; make it before any
 * stream capture.  Calls share the array: calls that overlap on the GPU race.
 * Allocates nothing. */
int klg_fwd_noalloc(const void* h_s, const void* h_t, const void* w, const uint8_t* mask, int64_t n_rows,
                    int64_t hidden, int64_t vocab, float inv_temp, int count_given, float* count, float* loss,
                    float* lse, float* row_kl, void* stream);

/* Scratch capacity of klg_fwd_noalloc, in floats. */
long long klg_fwd_noalloc_max_floats(void);

/* ---------------------------------------------------------------- backward
 * Replaces: autograd of train.py:202-210 (which stores bf16 [chunk, V] logits)
 * and, with the lm_head trainable, its weight gradient. */

/* Recommended workspace bytes for klg_bwd (a 4 KiB reserved header + a [n_rows, C]
 * bf16 dZ chunk of at most 512 MiB). */
int64_t klg_bwd_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab);

/* Vocab columns per backward chunk for a given workspace size (-1 if < 128). */
int64_t klg_bwd_chunk_cols(int64_t n_rows, int64_t vocab, int64_t workspace_bytes);

/* Pass 2: recomputes the logits chunk by chunk (never storing them) and
 * writes d_h_s [n_rows, H] fp32 (overwritten) and d_w [V, H] fp32 (overwritten).
 * grad = device scalar upstream gradient (NULL = 1).  Either output may be NULL
 * to skip it (the reference's lm_head is frozen: model.py:323-324). */
int klg_bwd(const void* h_s, const void* h_t, const void* w, const uint8_t* mask, const float* lse,
            const float* count, const float* grad, int64_t n_rows, int64_t hidden, int64_t vocab, float inv_temp,
            float* d_h_s, float* d_w, void* workspace, int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- training step
 * Forward and backward in one call (what the trainer does per diffusion chunk,
 * train.py:614-639: loss then backward).  Pass 1 computes only the two views'
 * log-sum-exps, on CTA pairs (tcgen05.mma.cta_group::2, 256 x 256 tiles); pass 2
 * recomputes the logits per vocab chunk, writes dZ, accumulates the KL cross term
 * sum_v p_v (z_t - z_s) per row on the way, and runs the dW / dH GEMMs; the loss is
 * formed at the end.  Gradients are for an upstream gradient *grad (NULL = 1).
 * row_kl (optional) holds KL for rows with mask set and 0 elsewhere. */

/* Recommended workspace bytes for klg_fwd_bwd. */
int64_t klg_fwd_bwd_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab);

/* dZ chunk width klg_fwd_bwd uses for a workspace of this size (-1 if too small). */
int64_t klg_fwd_bwd_chunk_cols(int64_t n_rows, int64_t hidden, int64_t vocab, int64_t workspace_bytes);

int klg_fwd_bwd(const void* h_s, const void* h_t, const void* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
                int64_t vocab, float inv_temp, int count_given, float* count, const float* grad, float* loss,
                float* lse, float* row_kl, float* d_h_s, float* d_w, void* workspace, int64_t workspace_bytes,
                void* stream);

/* klg_fwd_bwd that also records chunk_events[c] (cudaEvent_t handles, one per vocab chunk:
 * ceil(V / klg_fwd_bwd_chunk_cols(N, H, V, workspace_bytes)) of them) on the stream once chunk c's
 * GEMM is enqueued: from then on dW rows [c * cols, min(V, (c + 1) * cols)) are final, so a
 * row-sharded caller can all-reduce that slice on another stream while later chunks compute
 * (the bucketed, overlapped data-parallel gradient exchange). */
int klg_fwd_bwd_events(const void* h_s, const void* h_t, const void* w, const uint8_t* mask, int64_t n_rows,
                       int64_t hidden, int64_t vocab, float inv_temp, int count_given, float* count, const float* grad,
                       float* loss, float* lse, float* row_kl, float* d_h_s, float* d_w, void* workspace,
                       int64_t workspace_bytes, void* const* chunk_events, int n_events, void* stream);

/* Row-sharded training step with the dW exchange done over NVLink peer memory inside the step
 * (no counterpart in the reference; replaces klg_fwd_bwd + an all-reduce of dW): the dW GEMM
 * stores each 32-row block of this rank's partial dW into its owner's inbox (block b belongs to
 * rank b % world), then the owners sum their blocks in a fixed rank order and every rank copies
 * the sums into d_w, so d_w holds the sum over ranks on every rank when the stream reaches the
 * end of the call.  peer_buffers[world]: every rank's exchange buffer (klg_xr_buffer_bytes bytes,
 * zero-filled before the first call, addressable from this device: klg_xr_alloc / klg_xr_open),
 * the same on all ranks; epoch: 1 on the first call, +1 per call, the same on all ranks (it
 * orders the steps).  Every rank must make the call; a wait on a rank that does not arrive gives
 * up after ~1 s with KLG_STATUS_TIMEOUT_PEER (d_w is then invalid).  world in [2, 8]; bf16 path;
 * d_w required; loss and count as klg_fwd_bwd (count_given = 1 with the global count). */
int64_t klg_xr_buffer_bytes(int64_t vocab, int64_t hidden, int world);
int klg_fwd_bwd_xr(const void* h_s, const void* h_t, const void* w, const uint8_t* mask, int64_t n_rows,
                   int64_t hidden, int64_t vocab, float inv_temp, int count_given, float* count, const float* grad,
                   float* loss, float* lse, float* row_kl, float* d_h_s, float* d_w, void* workspace,
                   int64_t workspace_bytes, int world, int rank, void* const* peer_buffers, uint32_t epoch,
                   void* stream);

/* Exchange buffers over CUDA IPC (plain peer mappings, no multicast object): klg_xr_alloc
 * allocates and zero-fills `bytes` on `device` and writes its IPC handle (64 bytes) to
 * `handle`; every other rank opens it with klg_xr_open (its own device current); klg_xr_close
 * releases either (own = 1: the allocation, own = 0: a peer mapping). */
int klg_xr_alloc(int device, int64_t bytes, void** ptr, void* handle);
int klg_xr_open(int device, const void* handle, void** ptr);
int klg_xr_close(void* ptr, int own);

/* Test hook: the exchange's bounded wait on one GPU.  Runs the reduce step of the exchange on
 * `buffer` (klg_xr_buffer_bytes(vocab, hidden, 2) bytes, zero-filled) as rank 0 of 2 waiting for
 * an epoch no rank publishes: after ~1 s it sets KLG_STATUS_TIMEOUT_PEER and returns, the
 * context stays usable. */
int klg_selftest_xr_timeout(void* buffer, int64_t vocab, int64_t hidden, void* stream);

/* Leaves n_sms SMs of every device out of the persistent kernels' grids (0 = use all; at most
 * 64; process-wide, for launches planned after the call), so that communication kernels -- an
 * NCCL all-reduce of finished dW slices -- can run beside them. */
int klg_set_sm_reserve(int n_sms);

/* ---------------------------------------------------------------- fp32 inputs
 * The CPU-runnable configuration and the reference's fp32 teacher path (train.py:188-191)
 * compute in fp32; these variants keep fp32 fidelity on the bf16 tensor cores.  Each fp32
 * operand x is split into bf16 planes hi = bf16(x), lo = bf16(x - hi) and the planes are laid
 * side by side along H (hidden states [hi | hi | lo], lm_head [hi | lo | hi]), so a bf16
 * product over the 3H columns is h_hi w_hi + h_hi w_lo + h_lo w_hi: the logits carry ~2^-16
 * relative error before the fp32 accumulation.  dZ is kept as two bf16 planes (hi and lo) and
 * the dW / dH GEMMs add up both; the 3H-wide gradients are folded back to H.  Work is about
 * 3x (logits) to 6x (GEMMs) the bf16 path's.  Inputs h_s, h_t [N, H] and w [V, H] are fp32;
 * every other argument is as for klg_fwd_bwd / klg_fwd. */
int64_t klg_fwd_bwd_f32_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab);
int klg_fwd_bwd_f32(const float* h_s, const float* h_t, const float* w, const uint8_t* mask, int64_t n_rows,
                    int64_t hidden, int64_t vocab, float inv_temp, int count_given, float* count, const float* grad,
                    float* loss, float* lse, float* row_kl, float* d_h_s, float* d_w, void* workspace,
                    int64_t workspace_bytes, void* stream);
int64_t klg_fwd_f32_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab);
int klg_fwd_f32(const float* h_s, const float* h_t, const float* w, const uint8_t* mask, int64_t n_rows, int64_t hidden,
                int64_t vocab, float inv_temp, int count_given, float* count, float* loss, float* lse, float* row_kl,
                void* workspace, int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- training step in pieces
 * klg_fwd_bwd split at the points where a vocab-sharded step exchanges data (each rank holds
 * all rows and a slice of W's rows; the reference's loss is train.py:142-210 on one device):
 *   klg_lse_record   pass 1 over this W: one merged (m, S) record per row and view,
 *                    rec [2][2 * n_rows] = (m, S) in log2 units, rows 0..N-1 the student
 *                    view and N..2N-1 the teacher view            -> all-gather the records
 *   klg_lse_merge    n_rec such records (e.g. one per vocab shard) -> lse [2][n_rows]
 *   klg_pass2        with the global lse: dZ over this W, d_h_s (partial over the vocabulary:
 *                    all-reduce) and d_w (this W's rows, complete), and cross [n_rows], this
 *                    W's part of the KL cross term sum_v p_v (u_t - u_s) (log2 units) -> all-reduce
 *   klg_kl_loss      KL_i = ln2 (cross_i + lse_s,i - lse_t,i) for rows with mask set, and
 *                    loss = sum KL / count (0 when count == 0); row_kl may be NULL.
 * On one device with the whole W, klg_lse_record + klg_lse_merge (n_rec = 1) + klg_pass2 +
 * klg_kl_loss compute what klg_fwd_bwd computes. */
int64_t klg_lse_workspace_bytes(int64_t n_rows, int64_t vocab);
int klg_lse_record(const void* h_s, const void* h_t, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab,
                   float inv_temp, float* rec, void* workspace, int64_t workspace_bytes, void* stream);
int klg_lse_merge(const float* recs, int n_rec, int64_t n_rows, float* lse, void* stream);
int64_t klg_pass2_workspace_bytes(int64_t n_rows, int64_t hidden, int64_t vocab);
int klg_pass2(const void* h_s, const void* h_t, const void* w, const uint8_t* mask, const float* lse, const float* count,
              const float* grad, int64_t n_rows, int64_t hidden, int64_t vocab, float inv_temp, float* d_h_s,
              float* d_w, float* cross, void* workspace, int64_t workspace_bytes, void* stream);
int klg_kl_loss(const float* lse, const float* cross, const uint8_t* mask, int64_t n_rows, const float* count,
                float* loss, float* row_kl, void* stream);

/* ---------------------------------------------------------------- inference lm_head
 * The reference's sample_token (generate.py:40-78) on the lm_head output, without the
 * [N, V] logits (generate.py:161-188 computes the full logits first).  For each row of
 * h [N, H] (bf16): sample = 0 -> the argmax of z = h W^T (lowest index among equal
 * maxima, as torch.argmax); sample = 1 -> a draw from softmax(z * inv_temp) by the
 * Gumbel-max rule with a counter-based generator (seed, row, column) -- distributed like
 * torch.multinomial over the same probabilities, not the same stream.  Outputs: tokens
 * [N] int32, logit [N] = z of the chosen token, lse [N] = log sum exp(z * inv_temp), so
 * p(token) = exp(logit * inv_temp - lse).  top-k / top-p: klg_lm_head_sample_filtered. */
int64_t klg_lm_head_sample_workspace_bytes(int64_t n_rows, int64_t vocab);
int klg_lm_head_sample(const void* h, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab, float inv_temp,
                       int sample, uint64_t seed, int32_t* tokens, float* logit, float* lse, void* workspace,
                       int64_t workspace_bytes, void* stream);

/* Token selection with top-k / top-p filtering (generate.py:55-75) at temperature 1 / inv_temp,
 * still without [N, V] logits.  Two sweeps over W: the first gives each row's log-sum-exp and
 * its 32-column chunk maxima, from which a per-row threshold follows that no surviving logit is
 * below (with top-k on, the k-th largest chunk maximum, so that top-p then sees the whole top-k
 * set; for top-p alone, the chunk maximum at which the chunk maxima's own softmax mass passes
 * top_p); the second collects every logit at or above it (at most `cap`
 * per row).  A per-row kernel then applies the reference's rules exactly to those candidates
 * -- top-k keeps values >= the k-th largest, top-p keeps an entry while the mass strictly above
 * it is <= top_p (renormalised over the top-k survivors) -- and draws the Gumbel-max token
 * among the survivors with the unfiltered sampler's keys.  lse = log sum exp(z inv_temp) over
 * the survivors, so p(token) = exp(logit inv_temp - lse) is the reference's renormalised
 * probability.  *overflow (device int) is set when a row had more than `cap` candidates (its
 * token is then -1; call again with a larger cap, at most vocab).  top_k = 0 and top_p = 1
 * mean no filter.  Greedy selection has no filter (generate.py:52-53): use klg_lm_head_sample. */
int64_t klg_lm_head_sample_filtered_workspace_bytes(int64_t n_rows, int64_t vocab, int64_t cap);
int klg_lm_head_sample_filtered(const void* h, const void* w, int64_t n_rows, int64_t hidden, int64_t vocab,
                                float inv_temp, int top_k, float top_p, uint64_t seed, int64_t cap, int32_t* tokens,
                                float* logit, float* lse, int* overflow, void* workspace, int64_t workspace_bytes,
                                void* stream);

/* ---------------------------------------------------------------- row selection
 * The gathers of compute_kl_loss (train.py:124-139, 156-164) in one kernel:
 *   diff [B, nb*K, row] (the diffusion hidden states), ar [B, L, row] (AR hidden states),
 *   anchors [B, nb] int64, targets [B, nb*K] int64;
 *   row i = (b, blk, k), k = 1..K-1:  h_s[i] = diff[b, blk*K + k],
 *   h_t[i] = ar[b, clamp(anchors[b, blk] + k - 1, 0, L - 1)], valid[i] = targets[b, blk*K + k] != pad_id.
 * Rows are copied as bytes (row_bytes = H * element size, a multiple of 16).  The scatter is
 * the student gather's backward: d_diff[b, p] = d_hs[row of (b, p)], zeros at anchors (p % K == 0). */
int klg_gather_rows(const void* diff, const void* ar, const int64_t* anchors, const int64_t* targets, int64_t batch,
                    int64_t n_blocks, int64_t block, int64_t ar_len, int64_t row_bytes, int64_t pad_id, void* h_s,
                    void* h_t, uint8_t* valid, void* stream);
int klg_scatter_rows_grad(const void* d_hs, int64_t batch, int64_t n_blocks, int64_t block, int64_t row_bytes,
                          void* d_diff, void* stream);

/* ---------------------------------------------------------------- final RMSNorm prologue
 * For pre-norm hidden states: the backbone's final norm (model.py:493, `self.norm`, a
 * transformers LlamaRMSNorm) applied row by row, so the fused loss can take the states
 * before the norm.  x [N, H] bf16 (x_f32 = 0) or fp32 (x_f32 = 1); gamma [H] fp32 (the
 * norm weight; bf16 weights convert exactly).  r = 1 / sqrt(mean(x^2) + eps) (fp32);
 * y [N, H] bf16 = gamma * bf16(x r) rounded to bf16 for bf16 x -- the norm's own result
 * in a bf16 model -- and bf16(gamma * x r) for fp32 x.  rstd [N] (may be NULL) keeps r.
 * The backward gives dx [N, H] fp32 from dy [N, H] fp32 (the loss's dH):
 * dx = r gamma dy - (r^3 / H) x sum(gamma dy x).  The norm weight is frozen in the
 * reference (model.py:323-324), so no weight gradient is formed. */
int klg_rmsnorm_rows(const void* x, int x_f32, const float* gamma, int64_t n_rows, int64_t hidden, float eps, void* y,
                     float* rstd, void* stream);
int klg_rmsnorm_rows_bwd(const void* x, int x_f32, const float* gamma, const float* rstd, const float* dy,
                         int64_t n_rows, int64_t hidden, float* dx, void* stream);

/* ---------------------------------------------------------------- block-diffusion attention
 * The diffusion heads' attention (reference model.py:45-96 flex block mask, score_mod
 * model.py:435-446; the broken Triton version triton_kernels.py:18-83, API
 * triton_kernels.py:281-290), forward only: for query position p of block p / K, keys are
 * the AR cache rows 0..limits[b, p] (clamped to ar_len - 1; -1 = none) and the K rows of
 * its own block, scores scaled by `scale`, GQA (head h uses KV head h / (H / Hkv)).
 * The backward is klg_block_attn_bwd.
 *   q [B, H, Ld, 64], k_self / v_self [B, Hkv, Ld, 64] (bf16, contiguous),
 *   k_ar / v_ar: rows 0..ar_len-1 of a [B, Hkv, ar_stride, 64] bf16 cache,
 *   limits [B, Ld] int32; out [B, H, Ld, 64] bf16; lse [B, H, Ld] fp32 natural log (may be NULL).
 * head_dim 64; K a multiple of 16, <= 128; Ld a multiple of K.  The workspace is a token
 * 16 bytes (the key-range splits of a decode call combine on chip); the parameter stays so
 * that a later variant can use global scratch without an interface change. */
int64_t klg_block_attn_workspace_bytes(int64_t batch, int64_t heads, int64_t kv_heads, int64_t diff_len,
                                       int64_t block, int64_t ar_len, int64_t head_dim);
int klg_block_attn_fwd(const void* q, const void* k_self, const void* v_self, const void* k_ar, const void* v_ar,
                       int64_t ar_stride, const int32_t* limits, int64_t batch, int64_t heads, int64_t kv_heads,
                       int64_t diff_len, int64_t block, int64_t ar_len, int64_t head_dim, float scale, void* out,
                       float* lse, void* workspace, int64_t workspace_bytes, void* stream);

/* Backward of klg_block_attn_fwd (training the diffusion heads; the reference's Triton backward,
 * triton_kernels.py:73-141 and its autograd at 161-172, which the reference marks broken): for
 * the upstream gradient d_out [B, H, Ld, 64] bf16 and the forward's out (bf16) and lse (fp32,
 * natural log), writes d_q [B, H, Ld, 64] and the block keys' d_k_self / d_v_self
 * [B, Hkv, Ld, 64] (fp32; the dK / dV of a KV head sum over the query heads sharing it).  The
 * AR cache gets no gradient (it comes from the frozen backbone).  Same shapes and limits as the
 * forward; no workspace. */
int klg_block_attn_bwd(const void* q, const void* k_self, const void* v_self, const void* k_ar, const void* v_ar,
                       int64_t ar_stride, const int32_t* limits, const void* out, const float* lse, const void* d_out,
                       int64_t batch, int64_t heads, int64_t kv_heads, int64_t diff_len, int64_t block, int64_t ar_len,
                       int64_t head_dim, float scale, float* d_q, float* d_k_self, float* d_v_self, void* stream);

/* Number of AR key-range splits (the thread-block cluster size) klg_block_attn_fwd uses
 * for this shape on the current device; -1 for an unsupported shape. */
int klg_block_attn_splits(int64_t batch, int64_t heads, int64_t kv_heads, int64_t diff_len, int64_t block,
                          int64_t ar_len, int64_t head_dim);

/* Test hook (no counterpart in the reference): klg_block_attn_fwd with split `stall_split`
 * of every unit issuing no key/value loads, on a decode shape (splits >= 2).  That split's
 * operand wait runs out its bound (~1 s), sets a KLG_STATUS_TIMEOUT_* bit, and every CTA of
 * the cluster still meets at the cluster barriers and exits: the timeout path of a split
 * kernel ends with a status, not a hang.  The output is not meaningful. */
int klg_selftest_attn_split_stall(const void* q, const void* k_self, const void* v_self, const void* k_ar,
                                  const void* v_ar, int64_t ar_stride, const int32_t* limits, int64_t batch,
                                  int64_t heads, int64_t kv_heads, int64_t diff_len, int64_t block, int64_t ar_len,
                                  int64_t head_dim, float scale, void* out, float* lse, void* workspace,
                                  int64_t workspace_bytes, int stall_split, void* stream);

/* The logit z[i] = h[i] . W[tokens[i]] (fp32 accumulate of bf16 rows) of a token chosen
 * elsewhere -- with the lse of klg_lm_head_sample, exp(z * inv_temp - lse) is that token's
 * probability, the value the consensus step of generate.py:201-202 reads from the other
 * distribution's probs.  tokens [N] int32; a token outside [0, vocab) gives NaN. */
int klg_token_logit(const void* h, const void* w, const int32_t* tokens, int64_t n_rows, int64_t hidden, int64_t vocab,
                    float* z, void* stream);

/* fp32 -> bf16 conversion (round to nearest even) for fp32 callers. */
int klg_cast_f32_bf16(const float* in, void* out, int64_t n, void* stream);

/* out[i] = in[i] * (*g) (g a device float, or NULL for 1), as bf16 (out_bf16 = 1, round to
 * nearest even) or fp32, in one pass: the scaling of the saved dH / dW by the loss's upstream
 * gradient (torch.autograd.Function backward).  in and out 16-byte aligned. */
int klg_scale_cast(const float* in, const float* g, int64_t n, void* out, int out_bf16, void* stream);

/* ---------------------------------------------------------------- timing
 * Per-launch timing for benchmarks (the reference's counterpart is the manual
 * synchronize + perf_counter breakdown of train.py:541-547 and 676-685).
 * Between klg_trace_begin and klg_trace_end every kernel the library launches
 * (up to `capacity`) is bracketed by two CUDA events on its stream;
 * klg_trace_end waits for them and returns each launch's kind and duration. */
#define KLG_KIND_STATS 1     /* pass 1: both views' logits -> per-row partial records  */
#define KLG_KIND_DZ 2        /* pass 2: logit recompute -> dZ chunk                     */
#define KLG_KIND_GEMM 3      /* pass 2: dW chunk = dZ^T h_s and dH += dZ W_chunk        */
#define KLG_KIND_MERGE 4
#define KLG_KIND_FINALIZE 5
#define KLG_KIND_COUNT 6
#define KLG_KIND_CAST 7
#define KLG_KIND_ZERO 8      /* pass 2: zeroing of the fp32 dW / dH buffers            */
#define KLG_KIND_SAMPLE 9    /* inference: lm_head logits -> argmax / Gumbel-max sample   */
#define KLG_KIND_NORM 10     /* final RMSNorm of pre-norm rows, forward or backward       */
#define KLG_KIND_ATTN 11     /* block-diffusion attention, forward                        */
#define KLG_KIND_GATHER 12   /* row selection (gather) or its gradient scatter            */
#define KLG_KIND_XR 13       /* cross-rank dW exchange: owners' reduce, then the gather   */
int klg_trace_begin(int capacity);
int klg_trace_end(int* kinds, float* ms, int capacity, int* n);

#ifdef __cplusplus
}
#endif

#endif /* KLGEMM_H_ */
