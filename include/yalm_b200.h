/*
 * yalm_b200 — C ABI of the B200 (sm_100a) batch-1 decode engine for yalm .yalm checkpoints.
 *
 * The engine replaces the GPU side of yalm's `Model::forward` device dispatch
 * (src/model.cpp:479-494 of the yalm repository): the CUDA-graph backend `_forward_cuda`
 * (src/infer.cu:1274-1378) and the cooperative backend `yalm_coop_prepare` / `yalm_coop_forward`
 * (src/coop.h:5-6).  A yalm build binds it from a small shim: the shim fills
 * `yb_config` / `yb_weights` from yalm's `Config` and `Block` host pointers (the mmap'd .yalm
 * tensors, before `Model::cuda()` would upload them) and calls `yb_forward` with
 * `InferenceState::logits()`.
 *
 * Conventions
 *  - Every entry point that can fail returns 0 on success or a negative YB_E* code, and never
 *    aborts the process (yalm's CUDA_CHECK aborts, src/infer.cu:14-22).  The message of the last
 *    failure on the calling thread is available from yb_last_error().
 *  - All pointers in this header are host pointers unless the name says `_dev`.
 *  - fp16 values cross the ABI as uint16_t bit patterns (yalm's f16_t, src/codec.h:13).
 */
#ifndef YALM_B200_H
#define YALM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define YB_OK 0
#define YB_E_INVALID (-1)      /* bad argument or unsupported shape */
#define YB_E_CUDA (-2)         /* a CUDA runtime call failed */
#define YB_E_TIMEOUT (-3)      /* a bounded device-side wait ran out (status word set) */
#define YB_E_UNSUPPORTED (-4)  /* valid for yalm but not built here (MoE, fp32 weights) */

/* InferenceMode, src/model.h:43-46 */
#define YB_MODE_HYDRATE_KV_CACHE 0
#define YB_MODE_OUTPUT_LOGITS 1

/* Config, src/model.h:56-82 (fields the decode path uses).  act: 0 = GELU, 1 = SILU
 * (ActivationType, src/model.h:19-22).  weight_dtype in yalm's DType order (src/codec.h:15-25):
 * 1 = F16, or 3 = F8_E5M2 — the "fp8" dtype convert.py writes (convert.py:160, a plain cast to
 * float8_e5m2), which yalm's own runtime rejects (src/model.cpp:61-70); each E5M2 weight is the top
 * byte of the fp16 with the same value.  n_experts must be 0. */
typedef struct yb_config {
  int dim;
  int hidden_dim;
  int head_dim;
  int n_layers;
  int n_heads;
  int n_kv_heads;
  int vocab_size;
  int max_seq_len;
  int rotary_dim;
  int act;
  int n_experts;
  int weight_dtype;
  float rope_theta;
  float norm_eps;
  float qkv_clip; /* FLT_MAX when the checkpoint has no qkv_clip (src/model.cpp:59) */
} yb_config;

/* Host pointers to the tensors `Model` / `Block` hold before `cuda()` (src/model.h:249-264,
 * 276-281); per-layer arrays have n_layers entries.  Matrices are row-major exactly as in the .yalm
 * file: fp16 values, or for weight_dtype 3 one-byte E5M2 values (the pointers are then cast).  wcls
 * may equal token_embedding_table (tied embeddings, src/model.cpp:425-434). */
typedef struct yb_weights {
  const uint16_t* token_embedding_table; /* [vocab_size, dim] */
  const float* rms_final_weight;         /* [dim] */
  const uint16_t* wcls;                  /* [vocab_size, dim] */
  const float* const* rms_att_weight;    /* [n_layers] -> [dim] */
  const float* const* rms_ffn_weight;    /* [n_layers] -> [dim] */
  const uint16_t* const* wq;             /* [n_layers] -> [n_heads*head_dim, dim] */
  const uint16_t* const* wk;             /* [n_layers] -> [n_kv_heads*head_dim, dim] */
  const uint16_t* const* wv;             /* [n_layers] -> [n_kv_heads*head_dim, dim] */
  const uint16_t* const* wo;             /* [n_layers] -> [dim, n_heads*head_dim] */
  const uint16_t* const* w1;             /* [n_layers] -> [hidden_dim, dim] */
  const uint16_t* const* w2;             /* [n_layers] -> [dim, hidden_dim] */
  const uint16_t* const* w3;             /* [n_layers] -> [hidden_dim, dim] */
} yb_weights;

typedef struct yb_engine yb_engine;

/* ---------------------------------------------------------------- engine lifecycle */

/* Replaces Model::cuda() + InferenceState::cuda() (src/model.cpp:437-451, 342-361) and
 * yalm_coop_prepare (src/coop.h:5): uploads this rank's shard of the weights to `device`,
 * allocates the KV cache and activations, and records the per-step CUDA graphs.
 * tp_rank / tp_size: tensor-parallel position (tp_size 1 = single GPU).  For tp_size > 1 the
 * engines of all ranks must be joined with yb_tp_* before the first forward. */
int yb_create(const yb_config* cfg, const yb_weights* w, int device, int tp_rank, int tp_size, yb_engine** out);

/* Replaces Model::forward on a GPU device (src/model.cpp:479-494; _forward_cuda,
 * src/infer.cu:1274-1294; yalm_coop_forward, src/coop.h:6).  Runs one decode step for `token` at
 * position `pos` (ring buffer + attention sinks past max_seq_len, src/infer.cpp:489-494).
 * mode YB_MODE_OUTPUT_LOGITS: returns after the step completes, with vocab_size fp32 logits in
 * `logits` (InferenceState::logits(), any host memory).  YB_MODE_HYDRATE_KV_CACHE: only the KV
 * cache is updated; returns without waiting for the GPU, `logits` is ignored. */
int yb_forward(yb_engine* e, int token, int pos, int mode, float* logits);

/* One decode step in logits mode followed by yalm's sampler on the device, replacing
 * Model::forward + Sampler::sample (src/sampler.cpp:27-64): only the chosen id comes back to the
 * host (4 bytes instead of vocab_size fp32 logits).  temperature 0: greedy, the first index of the
 * maximum logit (sample_argmax, src/sampler.cpp:27-38).  temperature > 0: the first index whose
 * running sum of softmax(logits / temperature) reaches `coin` (yalm draws coin = rand() / RAND_MAX on
 * the host, src/sampler.cpp:55; pass the same value), else vocab_size - 1; the running sum is
 * formed in parallel, so the id can differ from yalm's sequential scan only when coin lies within
 * float rounding of a boundary.  Returns after the step; the logits stay on the device. */
int yb_forward_sample(yb_engine* e, int token, int pos, float temperature, float coin, int* next_token);

/* One decode step in logits mode followed by Sampler::sample_prob(target) on the device
 * (src/sampler.cpp:11-25, perplexity mode): *prob = exp(l_target - max) / sum_i exp(l_i - max). */
int yb_forward_prob(yb_engine* e, int token, int pos, int target, float* prob);

/* Replaces the prompt loop of yalm's run_completion (src/main.cpp:171-177: every prompt token
 * through Model::forward, HYDRATE_KV_CACHE but the last): tokens[0..n) at positions pos0 .. pos0+n-1
 * go through the model, filling the KV cache: all but the last token in one batched pass (tensor-core
 * GEMMs, causal attention over the cached and new slots), the last token as one decode step
 * (yb_forward), whose logits are written to `logits` when it is non-null.  Activations of the
 * batched pass are rounded to fp16 for the tensor cores, so the cache slots of the earlier prompt
 * tokens may differ from the per-token path by that rounding.  Engines or prompts the batched pass
 * does not cover (tensor parallel, fp8 weights, GELU, positions past the context, fewer than three
 * tokens) run the per-token steps.  Returns after completion. */
int yb_prefill(yb_engine* e, const int* tokens, int n, int pos0, float* logits);

/* Same step, logits left on the device (yb_logits_dev) and no host synchronisation: for
 * device-resident pipelines and benchmarks.  Follow with yb_sync before reading results. */
int yb_forward_async(yb_engine* e, int token, int pos, int mode);
int yb_sync(yb_engine* e);
const float* yb_logits_dev(yb_engine* e);
/* The CUDA stream the engine runs on (cudaStream_t). */
void* yb_stream(yb_engine* e);

/* Reads n cache slots [slot0, slot0 + n) of one layer / local kv head as fp16 bits in canonical
 * [slot][head_dim] order (yalm keeps K 16-tiled, src/model.h:14-17, and V as [head_dim][slot],
 * src/infer.cpp:304; this engine keeps both as [kv_head][slot][head_dim]). */
int yb_read_kv(yb_engine* e, int layer, int kv_head, int slot0, int n, uint16_t* k_out, uint16_t* v_out);

/* Which executor runs the steps: 0 = a CUDA graph of per-phase kernels chained with programmatic
 * dependent launch (replaces yalm's per-token CUDA graph, src/infer.cu:1296-1378), 1 = one
 * persistent cooperative kernel per step with bounded grid barriers between phases (replaces
 * yalm's cooperative kernel_forward, src/coop.cu:179-322).  The graph is the default (it measures
 * faster on B200); YB_EXECUTOR=persistent selects the persistent kernel when an instantiation exists
 * for the model shape. */
int yb_executor(yb_engine* e);

/* Diagnostics for an engine created with YB_TRACE=1: copies the last step's timeline, *grid rows
 * (CTAs) of *events %globaltimer stamps in ns (0 = not reached), into out (n entries); out = NULL
 * only reports *grid and *events.
 *  - persistent executor: per CTA, consumer start, arrive / release of every grid barrier in order,
 *    consumer end, producer end.
 *  - graph executor: 8 stamps per kernel of the step in launch order (per layer qkv, attention, wo,
 *    gate/up, w2; then the classifier in logits mode): for the matvecs j = 0 entry, 1 input vector
 *    loaded, 2 tensor-parallel all-reduce done (before 1), 3 last weight stage consumed, 4 epilogue
 *    done;
 *    for attention (row = blockIdx.y * gridDim.x + blockIdx.x) 0 entry, 7 early K/V copies
 *    issued, 1 inputs ready, 2 first K/V stage landed, 5 slots folded, 6 warp weights formed,
 *    3 CTA record written, 4 exit.  Rows beyond a kernel's grid stay 0. */
int yb_trace_read(yb_engine* e, unsigned long long* out, size_t n, int* grid, int* events);

/* Status word the kernels of the last step wrote (0 = healthy; bit 0 TMA-stage wait timed out,
 * bit 1 tensor-parallel peer wait timed out, bit 2 device-side argument check failed, bit 3 grid
 * barrier wait timed out). */
unsigned yb_status(yb_engine* e);
int yb_clear_status(yb_engine* e);

void yb_destroy(yb_engine* e);

/* Diagnostics: launches one of the engine's decode kernels `iters` times back to back on its own
 * weights and buffers (layer i mod n_layers for launch i, chained with programmatic dependent
 * launch as inside a step) and writes the mean device time per launch, from CUDA events on the
 * engine's stream, to *ms_per_launch.  which: 0 QKV, 1 attention, 2 wo, 3 gate/up, 4 w2,
 * 5 classifier.  Clobbers the activations and the KV slot of the last step's position, so call it
 * between sequences, not in the middle of one.  Single-GPU engines only. */
int yb_profile_kernel(yb_engine* e, int which, int iters, float* ms_per_launch);

/* Copies the message of the last failure on this thread into buf (NUL-terminated, truncated to
 * n bytes); returns the full message length. */
int yb_last_error(char* buf, int n);

/* ---------------------------------------------------------------- tensor parallelism
 * One process (or thread) per GPU.  Each rank exports an opaque blob describing its exchange
 * buffers (CUDA IPC handles), the blobs of all ranks are exchanged by the caller (e.g. an
 * all-gather over torch.distributed), and each rank imports all of them.  After that the engines
 * exchange partial sums over NVLink peer memory inside the wo / w2 kernels (no NCCL call on the
 * data path).  All ranks must then call yb_forward with identical (token, pos, mode) sequences. */
int yb_tp_export(yb_engine* e, void* blob, size_t blob_bytes, size_t* used);
int yb_tp_import(yb_engine* e, const void* blobs, size_t blob_stride);
size_t yb_tp_blob_bytes(void);

/* The slices yb_create uploads for rank tp_rank of tp_size (host arithmetic, no device needed), as
 * element ranges [begin, end): out8 = {Wq rows / Wo columns, Wk and Wv rows, W1 / W3 rows and W2
 * columns, classifier rows}.  The embedding and the norm weights are replicated.  No counterpart
 * in yalm, which runs on one GPU (src/model.cpp:442-443). */
int yb_tp_shard(const yb_config* cfg, int tp_rank, int tp_size, long long* out8);

/* ---------------------------------------------------------------- kernel-level entry points
 * Counterparts of yalm's test hooks (src/model.h:340-374: matmul_cuda, mha_cuda, ffn_cuda), with
 * the same argument meaning: host arrays in, host arrays out, synchronous.  They allocate device
 * memory per call and are meant for tests and tools, not for the decode loop. */

/* xout (d) = W (d, n) fp16 row-major @ x (n); n % 8 == 0.  matmul_cuda<f16_t>, src/model.h:359-360 */
int yb_matmul(float* xout, const float* x, const uint16_t* w, int n, int d);

/* multi-head attention over yalm's own cache layouts (kb 16-tiled, vb [n_kv][head_dim][max_seq_len]);
 * mha_cuda, src/model.h:348-355.  `att` is accepted for signature parity and not written. */
int yb_mha(float* xout, float* att, const uint16_t* kb, const uint16_t* vb, const float* q, int head_dim,
           int kv_len, int max_seq_len, int n_heads, int n_kv_heads);

/* xout (dim) = W2 @ (act(W1 @ x) * (W3 @ x)) with fp16 weights; ffn_cuda<f16_t>, src/model.h:368-374
 * (act: 0 GELU, 1 SILU). */
int yb_ffn(float* xout, const float* x, const uint16_t* w1, const uint16_t* w2, const uint16_t* w3, int hidden_dim,
           int dim, int act);

/* ---------------------------------------------------------------- device-pointer kernel launches
 * The individual decode kernels on caller-owned device buffers (for the kernel sweep and the
 * parity tests).  `stream` is a cudaStream_t (NULL = legacy default stream).  Asynchronous. */

/* y (rows) = W (rows, cols) @ x, or y += W @ x when accumulate != 0.  norm_w (cols) non-NULL:
 * x is RMS-normalised first with eps (src/infer.cpp:136-146).  Rows wider than one kernel covers
 * (fp16 beyond 14336 columns) run as equal column panels accumulated into y, as the engine runs
 * w2 at hidden_dim 28672; norm_w must then be NULL. */
int yb_gemv_dev(float* y, const float* x, const uint16_t* w, int rows, int cols, const float* norm_w, float eps,
                int accumulate, void* stream);

/* hb (hidden) = act(W1 @ xn) * (W3 @ xn) where xn = rmsnorm(x) if norm_w != NULL; w13 holds the
 * rows of W1 and W3 interleaved (row 2i = W1 row i, row 2i+1 = W3 row i). */
int yb_gateup_dev(float* hb, const float* x, const uint16_t* w13, int hidden, int dim, const float* norm_w, float eps,
                  int act, void* stream);

/* Fused QKV step of one layer: [q;k;v] = Wqkv ([(n_heads + 2 n_kv_heads) head_dim, dim], the rows of
 * Wq, Wk, Wv stacked) @ rmsnorm(x), clip, interleaved-pair RoPE at `pos`,
 * q -> q_out (fp32), k and v -> fp16 cache slot `kv_pos` of k_cache / v_cache
 * ([n_kv_heads][max_seq_len][head_dim]); when kv_sink > 0 also re-rotates the first kv_sink
 * cached keys by one position (src/infer.cpp:307-325).  inv_freq_dev: head_dim/2 floats
 * 1/theta^(2i/rotary_dim) in device memory. */
int yb_qkv_dev(float* q_out, uint16_t* k_cache, uint16_t* v_cache, const float* x, const uint16_t* wqkv,
               const float* norm_w, float eps, int dim, int n_heads, int n_kv_heads, int head_dim, int rotary_dim,
               int max_seq_len, int pos, int kv_pos, int kv_sink, float qkv_clip, const float* inv_freq_dev,
               void* stream);

/* Decode attention for all heads over cache slots [0, kv_len) of k_cache / v_cache
 * ([n_kv_heads][max_seq_len][head_dim] fp16): out (n_heads*head_dim) fp32.
 * scratch_dev: yb_attention_scratch_bytes(...) bytes of device memory (the cluster records of the
 * merge over several clusters of a kv head, and the kv heads' counters), zero-filled before its
 * first use and left zero by every call.  The first call per shape and device sets up its launch
 * (kernel attributes, the cluster size from the device's occupancy): make it outside stream
 * capture. */
int yb_attention_dev(float* out, const float* q, const uint16_t* k_cache, const uint16_t* v_cache, int n_heads,
                     int n_kv_heads, int head_dim, int max_seq_len, int kv_len, void* scratch_dev, void* stream);
size_t yb_attention_scratch_bytes(int n_heads, int n_kv_heads, int head_dim, int max_seq_len);
/* Diagnostics: the launch yb_attention_dev uses on the current device for this shape,
 * out20 = {CTAs per cluster, clusters per kv head, CTAs in the grid, dynamic shared memory bytes,
 * then for clusters of 1..16 CTAs the number the device holds at once}. */
int yb_attention_plan_info(int n_heads, int n_kv_heads, int head_dim, int max_seq_len, int* out20);

/* No counterpart in the yalm reference (it allocates with cudaMalloc wherever it needs memory).
 * yb_attention_dev for callers that must not allocate device memory when they call it — for
 * example a plugin whose host framework owns all device memory through its own allocator, or a
 * serving loop that forbids allocation after start-up to keep latency and memory use fixed.  Same
 * arguments and results as yb_attention_dev, without scratch_dev: the scratch lives in a fixed
 * YB_ATTENTION_NOALLOC_SCRATCH_BYTES array inside this library's device memory, which every GPU that
 * loads the library holds until the process exits.  Nothing is allocated or freed by the call.
 *  - Limit: yb_attention_scratch_bytes(n_heads, n_kv_heads, head_dim, max_seq_len) must not exceed
 *    YB_ATTENTION_NOALLOC_SCRATCH_BYTES (4 MiB: every shape of up to 256 heads of 128 fits); larger
 *    shapes return YB_E_INVALID with the sizes in yb_last_error().
 *  - The first call on each device looks up the array's device address (cudaGetSymbolAddress with
 *    that device current), and the first call for each shape on a device sets up its launch (a
 *    kernel attribute); make those first calls before any stream capture on the device.
 *  - All calls on a device share the one array, which keeps the previous call's contents (each
 *    call clears the part that must start at zero).  Calls whose executions overlap on the GPU, on
 *    different streams or host threads, race on it and give wrong results: order them on one
 *    stream or synchronise between them. */
#define YB_ATTENTION_NOALLOC_SCRATCH_BYTES (4u << 20)
int yb_attention_dev_noalloc(float* out, const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                             int n_heads, int n_kv_heads, int head_dim, int max_seq_len, int kv_len, void* stream);

/* Batched-prefill tensor-core GEMM on device buffers (no counterpart in yalm, which prefills one
 * token at a time, src/main.cpp:171-177): C[m][n] = sum_k A[m][k] * B[n][k] with A fp16 [M][K],
 * B fp16 [N][K] (a weight matrix as stored), fp32 accumulation; epi & 3: 0 stores C into out_f32,
 * 1 adds C to out_f32, 2 writes silu(C[m][2j]) * C[m][2j+1] to out_f16[m][j], 3 stores C as fp16
 * into out_f16; ldo is the output row stride in elements.  Flags: epi | 4 — A is two planes
 * [2][M][K], fp16 values and their fp16 remainders, both multiplied into C (fp32-like accuracy from
 * fp16 tensor cores); epi | 8 (with 2 or 3) — also write each fp16 output's remainder at
 * out_f16 + M * ldo.  K must be a multiple of 64 and N of 8. */
int yb_prefill_gemm_dev(float* out_f32, uint16_t* out_f16, const uint16_t* a, const uint16_t* b, int M, int N, int K,
                        int epi, int ldo, void* stream);

/* Batched-prefill causal attention on device buffers (the per-token loop of yalm's attention,
 * src/infer.cpp:218-250, for T new tokens at positions pos0 .. pos0 + T - 1 at once): q fp32
 * [T][n_heads * head_dim] (after RoPE), the head-major fp16 caches [n_kv_heads][max_seq_len][head_dim]
 * already holding slots 0 .. pos0 + T - 1; out fp16 [T][n_heads * head_dim].  Token t attends to
 * slots 0 .. pos0 + t. */
int yb_prefill_attention_dev(uint16_t* out, const float* q, const uint16_t* k_cache, const uint16_t* v_cache, int T,
                             int pos0, int n_heads, int n_kv_heads, int head_dim, int max_seq_len, void* stream);

/* Number of streaming multiprocessors the kernels size their grids for (device 0 if none set). */
int yb_num_sms(void);

#ifdef __cplusplus
}
#endif

#endif /* YALM_B200_H */
