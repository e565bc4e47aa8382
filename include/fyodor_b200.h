/* fyodor_b200.h - C ABI of the B200 provider for the Fyodor inference engine.
 *
 * The engine binds exactly one symbol, the provider vtable:
 *
 *   const nya_backend_interface *nya_cuda_backend(void);
 *
 * which replaces the reference provider's export in CUDA/cuda.c:457-462 and is
 * registered by backend/core/compute.c:7-9,25-27 when the engine is built with
 * NYA_ENABLE_CUDA. Its fields follow backend/include/compute_backend.h:12-29;
 * every return convention is the engine's (0 = output ready, -1 = decline or
 * failure, NULL plan = run the CPU reference).
 *
 * The fyb_* functions below are extensions for tools, tests and benchmarks
 * that need device-level access (no counterpart in the reference unless a
 * line says otherwise). They take plain pointers and sizes; "stream" is a
 * cudaStream_t passed as void* (NULL = the legacy default stream). Device
 * entry points return 0 on success, -1 for invalid arguments (nothing is
 * launched) and -2 for a CUDA launch failure.
 */
#ifndef FYODOR_B200_H
#define FYODOR_B200_H

#include "fyodor_b200_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Provider vtable. Replaces CUDA/cuda.c:457-462 (nya_cuda_backend). */
const nya_backend_interface *nya_cuda_backend(void);

/* Library identification (no counterpart in the reference). */
const char *fyb_version(void);
/* Number of CUDA devices visible to this process; 0 when none. */
int fyb_device_count(void);

/* ---- device-level kernels ---------------------------------------------- */

/* out[i] = value i of a GGUF tensor, bit-exact with the engine's
   nya_llm_tensor_value (backend/core/llm_quant.c:91-142). Device pointers. */
int fyb_dequantize(const void *weights, size_t count, unsigned type, float *out, void *stream);

/* Scratch needed by fyb_quant_matmul for one shape (bytes; 0 when none). */
size_t fyb_quant_matmul_workspace(size_t rows, size_t columns, unsigned type, size_t batch);

/* Y[b][r] = sum_k W[r][k] * X[b][k] on the device, the batched form of the
   engine's nya_compute_matmul_typed (backend/include/compute.h:80-83): W in
   GGUF row-major block storage, X batch-major [batch][columns], Y
   [batch][rows]. Q4_K/Q6_K run the tensor-core GEMV at batch 1-2 and the
   small-batch GEMM above it (up to 16 vectors per launch, every weight unit
   read once); Q8_0 with columns a multiple of 256 (and 16-byte aligned W and
   X) runs the bulk-staged Q8_0 kernel (up to 8 vectors per launch); every
   other case runs the type-generic kernel. `workspace` must hold
   fyb_quant_matmul_workspace() bytes: [counters][stream-K partials][repacked
   units][small-batch GEMM scratch], the counters zero before the first call
   (calls return them to zero). K-quant weights are repacked into the
   workspace on every call, so this entry point is for testing, not a hot
   loop (plans repack once). The layout depends on the device's SM count:
   use a workspace on the device it was sized for. */
int fyb_quant_matmul(const void *weights, size_t rows, size_t columns, unsigned type,
    const float *x, float *y, size_t batch, void *workspace, size_t workspace_bytes, void *stream);

/* fyb_quant_matmul in two halves (Q4_K/Q6_K only, -1 for other types): the
   repack of W into the workspace's units, once per weight matrix, then any
   number of products from the repacked workspace (the timed path of the
   matvec sweep). Same workspace size and results as fyb_quant_matmul. */
int fyb_quant_repack(const void *weights, size_t rows, size_t columns, unsigned type, void *workspace,
    size_t workspace_bytes, void *stream);
int fyb_quant_matmul_prepared(size_t rows, size_t columns, unsigned type, const float *x, float *y, size_t batch,
    void *workspace, size_t workspace_bytes, void *stream);

/* Decode attention over an fp16 KV cache for a ragged batch of sequences
   (no reference counterpart at this level; the engine's semantics are
   backend/core/llm_cpu.c:510-535 with an F32 cache).
   q   [nseq][heads][head_dim] f32, out [nseq][heads][head_dim] f32
   k,v per sequence s at k + s*seq_stride: [kv_heads][capacity][head_dim] f16
   lengths[s] = attended positions of sequence s (device array, 1..capacity).
   splits = context partitions per (sequence, kv head); 0 picks a default.
   workspace: fyb_attention_workspace() bytes, zero before the first call.
   With 2..64 query heads per KV head one CTA computes all of them on tensor
   cores (fp16 MMAs on hi/lo splits of q and of the probabilities, fp32
   accumulation), reading each K/V tile once. */
size_t fyb_attention_workspace(unsigned nseq, unsigned heads, unsigned kv_heads, unsigned head_dim, unsigned splits);
int fyb_attention_decode(const float *q, const void *k_cache, const void *v_cache, size_t seq_stride,
    const unsigned *lengths, unsigned nseq, unsigned heads, unsigned kv_heads, unsigned head_dim,
    unsigned capacity, float scale, float *out, unsigned splits, void *workspace, size_t workspace_bytes,
    void *stream);

/* Speculative verification: `queries` query rows per sequence (the draft
   tokens), causal within the draft (no counterpart in the reference, whose
   verification runs the drafts one decode step at a time,
   backend/core/llm_cpu.c:1274-1305). q and out are
   [nseq][queries][heads][head_dim]; lengths[s] counts sequence s's cached
   positions including its draft (>= queries), and query j attends positions
   0 .. lengths[s] - queries + j. workspace: fyb_attention_workspace(nseq *
   queries, ...) bytes, zero before the first call. nseq * queries <= 65535.
   When queries x (heads / kv_heads) <= 64 one CTA takes all draft rows of a
   KV head and reads each K/V tile once for them (the tensor-core kernel of
   fyb_attention_decode); otherwise every row streams the cache on its own. */
int fyb_attention_verify(const float *q, const void *k_cache, const void *v_cache, size_t seq_stride,
    const unsigned *lengths, unsigned nseq, unsigned queries, unsigned heads, unsigned kv_heads, unsigned head_dim,
    unsigned capacity, float scale, float *out, unsigned splits, void *workspace, size_t workspace_bytes,
    void *stream);

/* fyb_attention_decode without a workspace argument and without allocating
   anything (no counterpart in the reference). Same arguments and results as
   fyb_attention_decode; the scratch is a fixed array of
   FYB_ATTENTION_STATIC_SCRATCH_BYTES per device inside the library. Meant
   for callers that cannot allocate device memory where they call: a hook
   that runs under a device-memory budget it has already used up
   (NYA_CUDA_MEMORY_MIB), or a latency path that must not take cudaFree's
   implicit device synchronization.
   - The first call on a device (that device current) looks up the array's
     address; make that first call before any stream capture on the device.
   - Returns -3, launching nothing, when the problem needs more scratch than
     the array holds (fyb_attention_workspace() gives the need).
   - One array per device: calls that overlap in time on one device (other
     streams or threads) race on it and must be serialized by the caller.
   - The array is resident on every device that loads the library (4 MiB,
     outside the NYA_CUDA_MEMORY_MIB budget), and the address found at the
     first call assumes the device's primary context is never reset. */
#define FYB_ATTENTION_STATIC_SCRATCH_BYTES ((size_t)4 << 20)
int fyb_attention_decode_static(const float *q, const void *k_cache, const void *v_cache, size_t seq_stride,
    const unsigned *lengths, unsigned nseq, unsigned heads, unsigned kv_heads, unsigned head_dim,
    unsigned capacity, float scale, float *out, unsigned splits, void *stream);

/* ---- resident plans ---------------------------------------------------- */

/* Greedy decode entirely on the device: starting from `token` at `position`,
   run `steps` tokens, each taking the argmax of the previous logits (first
   index of the maximum, as nya_llm_sample with temperature 0 does,
   backend/core/llm_cpu.c:896-905). tokens_out[i] receives the i-th generated
   token. `plan` is a state returned by the vtable's plan_create. */
int fyb_plan_decode_greedy(void *plan, uint32_t token, size_t position, size_t steps, uint32_t *tokens_out);

/* Speculative verification (the engine's serial draft check,
   backend/core/llm_cpu.c:1274-1305, as one pass): count (1..16) draft tokens
   at positions [position, position + count) of a single-GPU plan's sequence
   (position <= the valid prefix), causal attention inside the draft, every
   weight read once for all of them; the logits of every draft position to
   logits [count][V] (suppressed ids -inf). The draft's K/V rows stay in the
   cache: the caller continues from the accepted prefix, whose later positions
   the next call rewrites. 0 / -1 invalid or no chunker (tensor-parallel
   shards, NYA_CUDA_CHUNKED_PREFILL=0) / -1 and a failed plan on a device
   error. */
int fyb_plan_verify(void *plan, const uint32_t *tokens, size_t count, size_t position, float *logits);

/* Times `steps` device-side greedy steps with CUDA events on the plan's
   stream (no host synchronization between steps); returns milliseconds or
   a negative value on failure. */
double fyb_plan_time_greedy(void *plan, uint32_t token, size_t position, size_t steps);

/* Kernel launches of one plan_token step: the request update plus the
   persistent decode kernel (2), or 3 + 5 per layer when the plan runs
   one kernel per operation. */
unsigned long long fyb_plan_launches_per_token(const void *plan);

/* Which decode step the plan runs: 0 one kernel per operation
   (NYA_CUDA_PERSISTENT=0 or an unsupported geometry), 1 the persistent
   kernel with CTA barriers between phases (default), 2 its dataflow form
   (NYA_CUDA_DATAFLOW=1: phases start per 256-column input block as its
   producers finish, no CTA barrier inside matrix phases; single GPU). -1 for
   a null plan. */
int fyb_plan_decode_form(const void *plan);

/* Average duration (ms) of each kernel class of one decode step measured
   with CUDA events around eager launches: out[0] matrix kernels, out[1]
   attention, out[2] other. Returns 0 on success. */
int fyb_plan_profile(void *plan, uint32_t token, size_t position, size_t steps, double *out);

/* Profiling of the persistent decode kernel (no reference counterpart): runs
   one decode step of `token` at `position` with per-CTA trace points and
   copies them to out[point * grid + cta] (globaltimer nanoseconds). Points
   per CTA: start; per layer, for the QKV, attention, O, gate/up and down
   phases, (CTA idle, dependency met) pairs, with a point after each input
   preparation and after the CTA's attention items; logits (idle, met,
   prepared); exit (idle, met). Returns the number of points per CTA and
   stores the grid in *grid_out, or -1 (plan without the persistent kernel,
   invalid arguments, out_count too small). With warp_out (may be NULL),
   also per-warp records of every GEMV phase: warp_out[((layer*5 + phase) *
   warps + warp) * 8 + k] (phase 0 QKV, 1 O, 2 gate/up, 3 down; layers*5 for
   the logits), k = 0 entry (ns), 1 SM clock cycles spent waiting for
   weights, 2 units computed (ns), 3 done (ns); then the default form's
   times (ns) after 4 the CTA barrier that follows the units, 5 the outputs
   of tiles shared between warps, 6 the fence, 7 the second CTA barrier; the
   dataflow form's 4 input preparation at phase entry done (ns), 5 cycles
   waiting for input blocks between units, 6 cycles in tile outputs;
   warp_count >= (layers*5 + 1) * grid * 16 * 8. The dataflow form has
   fewer CTA points (start; per layer the CTA idle and ready points before
   attention and the end of attention; exit idle and ready) and leaves the
   rest 0. */
long fyb_plan_trace(void *plan, uint32_t token, size_t position, unsigned long long *out, size_t out_count,
    unsigned *grid_out, unsigned long long *warp_out, size_t warp_count);

/* Average milliseconds of one stand-alone launch of a fused projection
   kernel of `layer` (which: 0 QKV+RoPE+KV append, 1 attention output,
   2 gate/up+SwiGLU, 3 down, 4 logits+argmax), timed over `reps` launches
   with CUDA events; *bytes receives the kernel's algorithmic bytes per
   launch (weights, input vector, norm weights, outputs). Timed launch i
   uses layer (layer + 1 + i) % layers, so with many layers consecutive
   launches read different weights (more bytes than L2 holds). */
double fyb_plan_time_projection(void *plan, unsigned layer, unsigned which, unsigned reps, size_t *bytes);

/* ---- batched decode (the engine's per-token step, reference
   CUDA/resident.inc:434-595 and backend/core/llm_cpu.c:424-578, applied to
   B sequences at once; the reference plan decodes one sequence) ----------
   fyb_batch_create: B (1..16) sequences of a resident plan's model, each with
   its own fp16 KV cache of the plan's capacity and its own position; they
   share the plan's weights (the plan must outlive the batch; single-GPU
   plans only). NULL if declined. Every step multiplies each weight once for
   all B sequences (batches of 9..16 on the tcgen05 small-batch GEMM).
   fyb_batch_step: one step of every sequence b at positions[b] with
   tokens[b] (position + 1 <= capacity); logits [B][V] (raw, no suppressed
   ids) and argmax [B] (first index of the maximum) copied out when
   non-null. 0 / -1 invalid / -2 device failure.
   fyb_batch_decode_greedy: `steps` greedy steps on the device from
   tokens / positions (each position + steps <= capacity); out [steps][B].
   fyb_batch_time_greedy: milliseconds per greedy step over `steps` graph
   replays (CUDA events) from tokens / positions (each position + steps <=
   capacity), after two untimed steps from the same start; < 0 on error.
   fyb_batch_launches_per_step: kernels in the last step enqueued. */
void *fyb_batch_create(void *plan, unsigned batch);
void fyb_batch_free(void *batch);
int fyb_batch_step(void *batch, const uint32_t *tokens, const uint32_t *positions, float *logits, uint32_t *argmax);
int fyb_batch_decode_greedy(void *batch, const uint32_t *tokens, const uint32_t *positions, size_t steps,
    uint32_t *out);
double fyb_batch_time_greedy(void *batch, const uint32_t *tokens, const uint32_t *positions, size_t steps);
unsigned long long fyb_batch_launches_per_step(const void *batch);

/* ---- tensor parallelism across processes (no reference counterpart) -----
   A process whose environment holds NYA_CUDA_TP_SIZE=N (2..8) and
   NYA_CUDA_TP_RANK=r (and NYA_CUDA_DEVICE for its GPU) creates plans that hold
   rank r's shard of the model: its H/N query and Hkv/N KV heads (rows of
   q/k/v, columns of the attention output), its FFN/N rows of gate/up and
   columns of down, and its V/N rows of the output head. The persistent decode
   kernel adds the ranks' partial attention-output and down rows over NVLink
   in every rank's exchange region (one exchange per attention block and one
   per MLP block), every rank gets the whole logits vector and the same greedy
   token. Before the first step each rank exports its exchange region with
   fyb_plan_tp_handle, the handles of all ranks are gathered (in rank order)
   by the caller, and every rank passes them to fyb_plan_tp_connect. The ranks
   must then run the same steps (plan_token, plan_prefill, greedy decoding)
   together; a rank that stops makes the others fail their next step after a
   bounded wait. plan_read_kv declines (a rank holds only its KV heads). */
#define FYB_IPC_HANDLE_BYTES 64
/* rank and size of the plan's shard (size 1 without tensor parallelism). */
int fyb_plan_tp_info(const void *plan, unsigned *rank, unsigned *size);
/* this rank's exchange region handle (FYB_IPC_HANDLE_BYTES bytes). */
int fyb_plan_tp_handle(void *plan, void *handle, size_t bytes);
/* opens the other ranks' regions; handles = count (= size) handles in rank order. */
int fyb_plan_tp_connect(void *plan, const void *handles, size_t count);
/* marks a connected plan unconnected again, so plan_token, plan_prefill and
   the greedy loop return -1 without launching: what every rank does when
   another rank could not create its plan or open the regions. */
int fyb_plan_tp_disconnect(void *plan);
/* connects plans that live in this one process (one thread per GPU, or
   several shards on one GPU): plans[j] is rank j's plan, count = size; the
   regions are used through their device pointers (peer access is enabled
   between different devices) instead of IPC handles. Connects `plan` only;
   call it once per plan. 0, -1 invalid arguments, -2 peer access refused. */
int fyb_plan_tp_connect_local(void *plan, void *const *plans, size_t count);
/* the plan's device error word: 0 none, 1 a bounded wait ran out (a peer or
   a producer never arrived), 2 non-finite logits, 4 an index out of range;
   -1 for a NULL plan. A plan with a non-zero word has failed. */
int fyb_plan_error(const void *plan);

/* ---- synthetic GGUF-layout models (no reference counterpart) -------------
   Builds an in-memory model in the engine's own binding layout
   (backend/core/llm_gguf.c:1013-1118): LLaMA tensors, block formats as
   given, random contents drawn from a seeded counter-based generator. */
typedef struct fyb_synth_config {
    uint32_t layers, embedding, heads, kv_heads, feed_forward, vocabulary, context;
    uint32_t matrix_type;   /* type of q/k/v/o/gate/up/down */
    uint32_t embed_type;    /* token_embd */
    uint32_t output_type;   /* output */
    float rope_base, epsilon;
    uint64_t seed;
    int norm_mode;          /* 0: all ones, 1: N(1, 0.01), 2: N(0, 1) */
    int threads;            /* host threads for filling; 0 = all cores */
    int centered;           /* Q4_K only: choose each group's min so its mean
                               weight is near zero (mins then are not uniform) */
    const char *path;       /* null: private memory. Otherwise the tensor bytes
                               live in this file, mapped shared: the first
                               process to create it fills it, later ones (same
                               configuration) wait until it is complete and map
                               it read-only, so ranks on one host share one copy,
                               as processes mapping one GGUF file do. */
} fyb_synth_config;
nya_llm_context *fyb_synth_create(const fyb_synth_config *config);
void fyb_synth_free(nya_llm_context *model);
/* Fill `bytes` of one tensor the way fyb_synth_create does (type-aware
   values: uniform quants, |N(0,1)|*0.01 fp16 scales). */
void fyb_synth_fill(void *data, size_t rows, size_t columns, uint32_t type, uint64_t seed, uint64_t stream_id);

#ifdef __cplusplus
}
#endif
#endif
