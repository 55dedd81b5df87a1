/*
 * veltrix_cuda.h — the C-ABI between Veltrix's C host code and the B200
 * kernels (library libveltrix_b200.so).
 *
 * Plain C types only: device pointers are `void *` / `float *` obtained from
 * cudaMalloc (or any allocator of device memory), streams are cudaStream_t
 * passed as `void *` (NULL = the legacy default stream).  Every function
 * returns a vx_error code (0 = VX_OK); vxc_error_string() gives the text of
 * the last failure on the calling thread.  There is no CPU fallback: with no
 * usable CUDA device every call fails with VX_ERR_UNSUPPORTED.
 *
 * Each entry point names the reference interface it replaces
 * (spear34000/veltrix-engine, file:line).
 */
#ifndef VELTRIX_CUDA_H
#define VELTRIX_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device & errors --------------------------------------------------- */

/* Select / initialise a CUDA device for the calling thread.  Fails with
 * VX_ERR_UNSUPPORTED when no CUDA device is present.  (No reference
 * counterpart: the reference is CPU-only, src/model.c:377-382 sets threads.) */
int vxc_device_init(int device);
int vxc_device_count(void);
/* Index of the calling thread's current CUDA device, or -1 without one. */
int vxc_device_current(void);
const char *vxc_error_string(void);
/* Read and clear the device-side error word that kernels set instead of
 * trapping (timeouts, out-of-range token ids).  Synchronises the device. */
int vxc_check_device_error(unsigned int *code_out);

/* Number of kernels this library has launched in this process (measurement
 * aid, no reference counterpart); a CUDA-graph replay counts the kernels it
 * holds. */
long long vxc_launch_count(void);

/* Per-stage device time of vxc_forward (measurement aid, no reference
 * counterpart).  While enabled, every eager (not graph-captured) forward
 * records CUDA events around its stages; vxc_profile_read synchronises,
 * writes the summed milliseconds of stage i to ms[i] for i < n, clears the
 * record and returns VXC_N_STAGES.  Stages: 0 embedding, 1 attention norm,
 * 2 QKV GEMV, 3 RoPE + KV write, 4 attention, 5 attention merge, 6 output
 * GEMV, 7 FFN norm, 8 gate/up GEMV, 9 SwiGLU, 10 down GEMV, 11 final norm +
 * LM head. */
#define VXC_N_STAGES 12
void vxc_profile_enable(int on);
int vxc_profile_read(double *ms, int n);

/* ---- quantised weight matrices ------------------------------------------ */

typedef struct vxc_qmat vxc_qmat;

/* Upload a GGUF-layout matrix of `rows` x `cols` (cols % 32 == 0) held in
 * host memory and repack it for the device (one record of quants + scales
 * per 128-row tile and 32-column block, records of a tile contiguous along
 * K).  type: 2 = Q4_0 (18-byte blocks), 8 = Q8_0 (34-byte blocks).
 * Replaces the reference's tensor load + whole-matrix dequant buffer
 * (src/gguf.c:236-287, src/model.c:74-87).
 * K-quant types 10..15 (Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K; cols % 256 == 0,
 * blocks of 84/110/144/176/210/292 bytes) are kept as GGUF super-blocks:
 * vxc_qgemv then decodes each weight as the reference does and sums in fp32
 * (the reference's blockwise GEMV, src/quantize.c:486-505; it needs no
 * workspace).  Nets may hold K-quant matrices and a K-quant token
 * embedding when every split is whole super-blocks and the parts fused into
 * one matrix (Q/K/V, gate/up) share one type. */
int vxc_qmat_create(int type, const void *host_blocks, int rows, int cols, vxc_qmat **out);
/* Decoded weights of a K-quant matrix, fp32 [rows][cols] in device memory,
 * bit for bit the reference's vx_dequantize_row_* for the type. */
int vxc_kquant_dequant(const vxc_qmat *w, float *y, void *stream);
void vxc_qmat_destroy(vxc_qmat *w);
int vxc_qmat_shape(const vxc_qmat *w, int *type, int *rows, int *cols);

/* Bytes of scratch vxc_qgemv (and vxc_qgemv_simt) needs for M activation
 * rows: the split-K partial sums and, above 16 rows, the activation image
 * and its prescales (from 64 rows: the image in slabs of 256 rows, the
 * prescales and the GEMM's K-slice sums).  Nothing in it has to be
 * initialised. */
size_t vxc_qgemv_workspace_bytes(const vxc_qmat *w, int M);

/* y[m][r] = sum_k W[r][k] * x[m][k] for m < M (fp32 in, fp32 out, device
 * pointers, row-major with leading dimensions cols and rows).  Q4_0 follows
 * the reference's interleaved nibble order.  Replaces vx_gemv_q4_0
 * (src/quantize.c:728-750), vx_gemv_q4_0_avx2 (src/simd/avx2.c:311-370) and
 * apply_gemv's Q8_0 path (src/model.c:234-244), batched over M rows.
 * 1-2 rows run on the CUDA cores, up to 63 on the tensor-core GEMV, from 64
 * on the tensor-core GEMM (weights converted once per 256-row slab; a row's
 * result does not depend on the other rows).
 * `workspace` must hold vxc_qgemv_workspace_bytes(w, M) bytes (may be NULL
 * when that is 0). */
int vxc_qgemv(const vxc_qmat *w, const float *x, int M, float *y, void *workspace,
              size_t workspace_bytes, void *stream);

/* Same product through the exact CUDA-core kernel (fp32 FMA, no tensor
 * cores); kept as an independent second implementation for tests. */
int vxc_qgemv_simt(const vxc_qmat *w, const float *x, int M, float *y, void *workspace,
                   size_t workspace_bytes, void *stream);

/* vxc_qgemv without a caller-provided workspace, for callers that cannot
 * allocate device memory (a host application that owns the device memory
 * budget and forbids libraries to call cudaMalloc, or latency-bound code that
 * cannot afford cudaMalloc's device synchronisation).  No reference
 * counterpart.  The scratch is a static device array of
 * VXC_QGEMV_NOALLOC_BYTES (8 MiB) held by every GPU that loads the library;
 * shapes whose vxc_qgemv_workspace_bytes exceeds it are rejected (-4, see
 * vxc_error_string).  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  Calls share the array: calls that overlap on the GPU race. */
#define VXC_QGEMV_NOALLOC_BYTES (8u << 20)
int vxc_qgemv_noalloc(const vxc_qmat *w, const float *x, int M, float *y, void *stream);

/* ---- device model ---------------------------------------------------------- */

/* A host tensor in GGUF layout: type 0 = F32, 2 = Q4_0, 8 = Q8_0; `rows` x
 * `cols` with cols the contiguous (ne0) dimension.  data == NULL = absent. */
typedef struct {
    int type;
    int rows, cols;
    const void *data;
} vxc_tensor_view;

typedef struct {
    vxc_tensor_view attn_norm, wq, wk, wv, wo, ffn_norm, wg, wu, wd;
} vxc_layer_views;

/* Llama-family hyper-parameters (reference vx_model_config,
 * include/veltrix.h:80-102; rope_theta as read by src/gguf.c:533). */
typedef struct {
    int n_layers, n_heads, n_kv_heads, n_embd, n_head_dim, n_ff, n_vocab;
    int max_pos;          /* largest position the RoPE table covers */
    float rope_theta;
} vxc_net_config;

typedef struct vxc_net vxc_net;
typedef struct vxc_seqs vxc_seqs;

/* Upload a model (weights stay resident; QKV and gate/up are fused per
 * layer).  Replaces the reference's load + consolidate step
 * (src/model.c:18-111) for the device. */
int vxc_net_create(const vxc_net_config *cfg, const vxc_tensor_view *tok_embd, const vxc_tensor_view *out_norm,
                   const vxc_tensor_view *output, const vxc_layer_views *layers, vxc_net **out);
void vxc_net_destroy(vxc_net *net);

/* ---- tensor parallelism (one process per GPU, NCCL over NVLink) ----------- */

/* A communicator over `world` GPUs, one per process.  Rank 0 makes the id
 * (VXC_TP_ID_BYTES bytes) and hands it to the others out of band. */
typedef struct vxc_tp vxc_tp;
#define VXC_TP_ID_BYTES 128
int vxc_tp_unique_id(void *id_out);
int vxc_tp_create(const void *id, int rank, int world, vxc_tp **out);
void vxc_tp_destroy(vxc_tp *tp);
/* Upload this rank's shard of a model split over tp's GPUs (Megatron-style):
 * rank r keeps heads [r*H/w, (r+1)*H/w) of Q, the matching KV heads, rows
 * [r*F/w, ...) of gate/up, the matching columns of wo and wd, and rows
 * [r*V/w, ...) of the LM head; embeddings and norms are replicated.  Each
 * forward then sums the wo and wd outputs over the GPUs (all-reduce) and
 * gathers the logits (all-gather), so every rank sees the full logits.
 * H, KV heads, n_ff and n_vocab must divide by the world size.  tp == NULL
 * is vxc_net_create.  The net borrows tp, which must outlive it. */
/* The split vxc_net_create_tp applies, for inspection and host-side tests
 * (no device needed): out[8][4] = {first row, rows, first column, columns}
 * of this rank's slice of Wq, Wk, Wv, Wo, W_gate, W_up, W_down and the LM
 * head, in elements of the GGUF [rows][cols] matrices. */
int vxc_tp_shard_ranges(const vxc_net_config *cfg, int rank, int world, int *out);
int vxc_net_create_tp(const vxc_net_config *cfg, const vxc_tensor_view *tok_embd, const vxc_tensor_view *out_norm,
                      const vxc_tensor_view *output, const vxc_layer_views *layers, const vxc_tp *tp,
                      vxc_net **out);
/* A net whose weights are generated on the device: N(0, 0.02) from
 * Philox4x32-10 keyed by (seed, tensor, element) and quantised to `wtype`
 * (2 Q4_0, 8 Q8_0), norms 1.0 -- the weights vx_synth_write_gguf would
 * write for the same configuration and seed, up to the device's rounding of
 * double-precision log/sqrt/cos/sin.  With tp, only this GPU's shard is
 * generated.  For timing runs of shapes whose checkpoint files would be tens
 * of GB. */
int vxc_net_create_synth(const vxc_net_config *cfg, int wtype, uint64_t seed, const vxc_tp *tp, vxc_net **out);
int vxc_net_config_get(const vxc_net *net, vxc_net_config *cfg);
/* Device bytes of weights read by one forward pass (all matrices + norms). */
size_t vxc_net_weight_bytes(const vxc_net *net);

/* KV cache for n_slots independent sequences of up to max_ctx positions
 * (fp32, [layer][slot][kv head][pos][head_dim] — reference src/model.c:404-411 keeps
 * one [layer][n_ctx][kv_dim] cache per model) plus work buffers for up to
 * max_rows rows per forward call. */
int vxc_seqs_create(const vxc_net *net, int n_slots, int max_ctx, int max_rows, vxc_seqs **out);
void vxc_seqs_destroy(vxc_seqs *s);

/* Batched forward (reference vx_model_forward, src/model.c:391-628, for many
 * tokens and sequences at once).  Rows come in n_groups groups of
 * rows_per_group consecutive tokens; group g belongs to sequence slot
 * d_slot[g] and its row t sits at position d_pos[g] + t.  K/V of every row
 * are written into the slot's cache before attention, so each row attends to
 * positions 0..its own position (causal within the group).  Logits are
 * produced for the rows listed in d_logit_rows (n_logit_rows of them) into
 * d_logits[n_logit_rows][n_vocab].  All d_* pointers are device memory;
 * nothing is copied to the host, so the call can be captured in a CUDA graph.
 * Rows with an out-of-range token or position raise the device error word. */
int vxc_forward(vxc_seqs *s, const int *d_tokens, const int *d_slot, const int *d_pos, int n_groups,
                int rows_per_group, const int *d_logit_rows, int n_logit_rows, float *d_logits, void *stream);

/* Host-buffer form of vxc_forward for one sequence (the drop-in path of
 * vx_model_forward): n_tokens host tokens at positions pos0.. of `slot`;
 * the logits of the last token go to h_logits (n_vocab floats).  Processes
 * the tokens in chunks of max_rows and synchronises. */
int vxc_forward_host(vxc_seqs *s, int slot, int pos0, const int *h_tokens, int n_tokens, float *h_logits);

/* Greedy decoding of one sequence (the loop of the reference's CLI,
 * src/main.c:283-324): forward the prompt at positions pos0.., then emit the
 * argmax token (first index of the maximum, src/main.c:307-311) and forward
 * it, until max_tokens are emitted or the argmax is eos_id (not emitted;
 * eos_id < 0: none).  The reference forwards the last prompt token a second
 * time before its loop (src/main.c:283,300-304); this loop does not.  Each
 * token is one CUDA-graph replay with no host round trip.  *n_out = tokens
 * written to h_out; *pos_out = positions now cached (the last emitted token
 * is not yet in the cache).  Returns 0 or an error code. */
int vxc_greedy_generate(vxc_seqs *seqs, int slot, int pos0, const int *h_prompt, int n_prompt, int *h_out,
                        int max_tokens, int eos_id, int *n_out, int *pos_out);

/* ---- sampling ----------------------------------------------------------------
 * Canonical sampler shared with the CPU oracle (bit-exact given the same fp32
 * logits): T <= 0 is greedy (first maximum, reference src/speculative.c:93-98);
 * otherwise W_v = trunc(exp((l_v - max)/T) * 2^32) with a fixed exp, and a
 * token is drawn as the first v whose prefix sum of W exceeds
 * floor(sum(W) * u24 / 2^24), u24 = Philox4x32-10(seed; pos, seq, purpose) >> 8.
 */

/* One token per row of logits[n_rows][V] (device) into tokens[n_rows]
 * (device), row r using Philox counter (pos[r], seq[r], purpose);
 * n_rows <= 65535.
 * Replaces sample_top_p / sample_greedy (src/speculative.c:35-98) with
 * top_p = 1. */
int vxc_sample_rows(const float *logits, int n_rows, int V, float temp, uint64_t seed, const int *d_pos,
                    const int *d_seq, unsigned int purpose, int *d_tokens, void *stream);

/* Scratch bytes vxc_accept needs for n_seq sequences of k draft tokens
 * (0 with the current kernel, which keeps its state on chip; callers pass
 * what this returns, and workspace may then be NULL). */
size_t vxc_accept_workspace_bytes(int n_seq, int k);

/* Fused acceptance for n_seq sequences (reference verify_draft,
 * src/speculative.c:178-236, restated as standard speculative sampling):
 * P = target logits (row i of sequence s at P + s*p_seq + i*p_pos, i <= k),
 * Q = draft logits (row i at Q + s*q_seq + i*q_pos, i < k), draft tokens
 * d[s*k + i].  Draft token i of sequence s sits at absolute position
 * pos0[s] + i and uses Philox counters (pos0[s]+i, seq_id[s], ACCEPT /
 * RESAMPLE).  Outputs n_acc[s] in 0..k and next[s] (the correction token,
 * or the bonus token drawn from row k when all k are accepted).  One kernel
 * launch (one thread-block cluster per sequence); all pointers are device
 * memory; k <= 64 and n_seq <= 65535. */
int vxc_accept(const float *P, long long p_seq, long long p_pos, const float *Q, long long q_seq,
               long long q_pos, const int *d, int n_seq, int k, int V, float temp, uint64_t seed,
               const int *seq_id, const int *pos0, int *n_acc, int *next, void *workspace,
               size_t workspace_bytes, void *stream);

/* ---- device speculative-decoding engine --------------------------------------- */

typedef struct vxc_spec vxc_spec;

typedef struct {
    long long rounds;      /* draft+verify rounds run */
    long long drafted;     /* draft tokens proposed (sum over sequences) */
    long long accepted;    /* draft tokens accepted */
    long long emitted;     /* tokens written to the outputs */
    double prefill_ms;     /* device time of the prompt pass */
    double decode_ms;      /* device time of the round loop */
} vxc_spec_stats;

/* Engine for up to n_seq concurrent sequences of max_ctx positions, k draft
 * tokens per round; keeps KV caches for both models. */
int vxc_spec_create(const vxc_net *target, const vxc_net *draft, int n_seq, int k, int max_ctx, vxc_spec **out);
void vxc_spec_destroy(vxc_spec *e);

/* Generate up to max_new tokens for each of n_seq sequences (host buffers:
 * prompts concatenated, prompt_len[n_seq], seq_id[n_seq] = Philox sequence
 * ids; out[n_seq][max_new], counts[n_seq]).  Replaces
 * vx_speculative_generate (src/speculative.c:238-294) for a batch; the
 * whole round loop (k draft steps, one (k+1)-row verify, fused acceptance,
 * commit) runs on the device as one CUDA graph per round. */
int vxc_spec_generate(vxc_spec *e, const int *prompts, const int *prompt_len, const int *seq_id, int n_seq,
                      int max_new, float temp, uint64_t seed, int *out, int *counts, vxc_spec_stats *stats);

/* Measurement hook (no reference counterpart): after a generate call, re-run
 * one piece of the last round `reps` times and return its average device
 * time in *ms: which = 0 the (k+1)-row target verify forward, 1 one draft
 * step, 2 the fused acceptance kernel.  *kv_bytes (may be NULL) receives the
 * K/V cache bytes one such forward reads and writes.  The committed tokens
 * are not changed. */
int vxc_spec_probe(vxc_spec *e, int which, int reps, double *ms, double *kv_bytes);

#ifdef __cplusplus
}
#endif

#endif
