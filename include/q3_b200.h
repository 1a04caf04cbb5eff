/*
 * q3_b200.h - C ABI of the B200 (sm_100a) Qwen3 forward pass.
 *
 * Drop-in boundary for the hot path of asriva32/Qwen3.cpp: the C++ surface of that project's
 * include/inference.h (class Qwen3, class Block, the free kernels RmsNorm/MatMul/...,
 * Sampler::Greedy) re-expressed as plain C entry points over plain pointers and sizes. Each
 * declaration names the reference interface it replaces. The C++ classes in
 * include/inference_b200.h are a thin layer over these functions.
 *
 * Conventions
 *  - Every function returns q3_status. Codes 1-3 map one to one onto the exception types the
 *    reference throws (std::runtime_error, std::invalid_argument, std::out_of_range); the
 *    message of the last failure on the calling thread is q3_last_error().
 *  - "_host" pointers are caller-owned host memory; all other data pointers are device pointers.
 *  - A model or block handle owns its device memory (weights, KV cache, workspace) and one CUDA
 *    stream; calls on a handle block until their work on that stream is done. Handles are not
 *    thread-safe (the reference's Qwen3 and Block are not either).
 *  - bf16 values travel as their raw uint16_t bit patterns.
 */
#ifndef Q3_B200_H
#define Q3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum q3_status {
    Q3_OK = 0,
    Q3_ERR_RUNTIME = 1,          /* std::runtime_error: file/format errors, CUDA failures */
    Q3_ERR_INVALID_ARGUMENT = 2, /* std::invalid_argument: bad config, sizes, null pointers */
    Q3_ERR_OUT_OF_RANGE = 3,     /* std::out_of_range: token id, position or KV range */
    Q3_ERR_DEVICE_TIMEOUT = 5    /* a bounded device-side wait gave up (reported, not hung) */
} q3_status;

/* Config (include/inference.h:66-90). max_seq_len is the runtime context once a model is
 * loaded (Qwen3::InitializeInference overwrites it, src/inference.cpp:534). */
typedef struct q3_config {
    int32_t dim, hidden_dim, head_dim, n_layers, n_heads, n_kv_heads, vocab_size, max_seq_len;
    int32_t bos_token_id, eos_token_id, rotary_dim;
    float rope_theta, norm_eps;
    int32_t tie_word_embeddings, attention_bias, qk_norm;
} q3_config;

/* GenerationStats (include/inference.h:209-219); seconds are host wall clock. */
typedef struct q3_generation_stats {
    size_t prompt_tokens, generated_tokens;
    double prefill_seconds, decode_seconds;
    int32_t stopped_on_eos, reached_token_limit;
} q3_generation_stats;

typedef struct q3_model q3_model;
typedef struct q3_block q3_block;

const char* q3_last_error(void);
const char* q3_version(void);

/* ------------------------------------------------------------------ whole model (class Qwen3) */

/* Qwen3::Qwen3(path, context_length) + InitializeInference (src/inference.cpp:445-510, :529-581):
 * parses Qwen3.bin (the convert.py layout) and uploads every tensor into one HBM arena on
 * `device`. Same validation and error kinds as the reference loader. */
q3_status q3_model_load(const char* path, int context_length, int device, q3_model** out);
void q3_model_free(q3_model* model);

/* Qwen3::GetConfig (src/inference.cpp:512-514). */
q3_status q3_model_config(const q3_model* model, q3_config* out);
/* Qwen3::GetTensorIndex().size() (src/inference.cpp:516-518). */
q3_status q3_model_tensor_count(const q3_model* model, int* out);

/* Config::arch / dtype / act_type (include/inference.h:66-90), the metadata strings of the file.
 * key is "arch", "dtype" or "act_type"; *length (nullable) receives the string length; buf
 * (nullable) receives the NUL-terminated string and needs length+1 bytes. */
q3_status q3_model_metadata(const q3_model* model, const char* key, char* buf, size_t capacity,
                            size_t* length);

/* TensorInfo (include/inference.h:30-36) of one record of the file; dtype uses the reference's
 * TensorDType codes (1 f32, 3 bf16, 4 u8, 5 i32); data_offset is the payload's byte offset in
 * the file. Unknown names fail like Qwen3::LoadTensor ("Tensor not found", runtime error). */
typedef struct q3_tensor_info {
    uint32_t dtype, rank;
    uint64_t shape[8];
    uint64_t data_offset, byte_size;
} q3_tensor_info;
/* Name of record `index` (0 .. tensor_count-1, file order): the keys of Qwen3::GetTensorIndex()
 * (src/inference.cpp:516-518). *length and buf as in q3_model_metadata. */
q3_status q3_model_tensor_name(const q3_model* model, int index, char* buf, size_t capacity,
                               size_t* length);
/* Qwen3::GetTensorIndex().find(name) (src/inference.cpp:516-518). */
q3_status q3_model_tensor_info(const q3_model* model, const char* name, q3_tensor_info* out);
/* Qwen3::LoadTensor<T>(name) (include/inference.h:289-305, LoadTensorBytes at
 * src/inference.cpp:307-317): copies the payload (byte_size bytes) to host; a record whose dtype
 * is not expected_dtype fails with "Tensor dtype mismatch" (runtime error). */
q3_status q3_model_load_tensor(const q3_model* model, const char* name, uint32_t expected_dtype,
                               void* host, size_t capacity);

/* Qwen3::ResetInference (src/inference.cpp:583-590): zeroes every KV cache. */
q3_status q3_reset(q3_model* model);

/* Qwen3::ForwardToken (src/inference.cpp:592-637): one token at absolute position `pos`
 * (attention-sink ring buffer once pos >= context), logits[vocab_size] to logits_host. */
q3_status q3_forward_token(q3_model* model, int32_t token, int pos, float* logits_host);

/* Qwen3::ForwardToken with the reference's return convention (`const std::vector<float>&`,
 * include/inference.h:227-229, src/inference.cpp:592-637): *logits points at vocab_size floats in
 * a model-owned pinned host buffer, valid until the next call on this model. */
q3_status q3_forward_token_ref(q3_model* model, int32_t token, int pos, const float** logits);

/* Qwen3::ForwardToken followed by Sampler::Greedy on its logits (the two calls of each step of
 * Qwen3::Generate, src/inference.cpp:680-683, :703-709): *logits as q3_forward_token_ref, and
 * *next_token = the index of their first maximum, computed on the device. */
q3_status q3_forward_token_greedy(q3_model* model, int32_t token, int pos, const float** logits,
                                  int32_t* next_token);

/* ForwardToken with debug taps: hidden_host[(n_layers+1)*dim] receives the embedding row and
 * the hidden state after each layer (the per-layer view of src/inference.cpp:615-617). Either
 * output may be NULL. */
q3_status q3_forward_token_layers(q3_model* model, int32_t token, int pos, float* hidden_host,
                                  float* logits_host);

/* Row kv_pos (ring slot) of layer `layer`'s bf16 KV cache, n_kv_heads*head_dim values each in
 * the reference layout of KVCache (include/inference.h:140-161). */
q3_status q3_kv_row(q3_model* model, int layer, int kv_pos, uint16_t* k_host, uint16_t* v_host);

/* Batched prefill of n prompt tokens at positions pos0..pos0+n-1 (replaces the token-at-a-time
 * loop of Qwen3::Generate, src/inference.cpp:669-671). Leaves the KV cache as n ForwardToken
 * calls would. last_logits_host (nullable) receives the logits of the last token;
 * next_token_host (nullable) its greedy argmax. */
q3_status q3_prefill(q3_model* model, const int32_t* ids_host, int n, int pos0,
                     float* last_logits_host, int32_t* next_token_host);

/* q3_prefill with debug taps: hidden_host[(n_layers+1)*dim] (nullable) receives the hidden state
 * of the LAST prompt token before the first layer and after every layer. */
q3_status q3_prefill_layers(q3_model* model, const int32_t* ids_host, int n, int pos0,
                            float* hidden_host, float* last_logits_host, int32_t* next_token_host);

/* Prefill paths (no reference counterpart: the reference prefills token by token). BATCHED runs
 * every projection as a tensor-core contraction over all prompt tokens (tcgen05, fp32
 * accumulation) and causal attention over the paged cache; it is used when the model shape
 * allows it (head_dim 128, two query heads per KV head) and pos0 + n <= context, and is the
 * default. TOKENWISE feeds the prompt through the decode path one token at a time. */
enum { Q3_PREFILL_TOKENWISE = 0, Q3_PREFILL_BATCHED = 1 };
q3_status q3_model_set_prefill_path(q3_model* model, int path);
/* The path q3_prefill takes for prompts that fit below the context. */
q3_status q3_model_prefill_path(const q3_model* model, int* path);
/* Operand precision of the batched prefill (also used by q3_batch_add). F16 (the default): fp16
 * copies of the weights (the bf16 values, exact in their range; made on first use, +0.88 GB for
 * Qwen3-0.6B) and fp16 activations, the [wq;wk;wv] input as an fp16 hi + lo pair, attention on
 * fp16 copies of the cache rows (+ the cache's size); decode after a long prompt then agrees with
 * the reference as decode after a short one does. BF16: one bf16 rounding per activation operand
 * (8 significant bits against 11), no extra memory. The tensor-core rate is the same. */
enum { Q3_PREFILL_BF16 = 0, Q3_PREFILL_F16 = 1 };
q3_status q3_model_set_prefill_precision(q3_model* model, int precision);
q3_status q3_model_prefill_precision(const q3_model* model, int* precision);

/* n_steps greedy decode steps driven on the device (the loop of src/inference.cpp:679-690 with
 * stop_on_eos = false, i.e. `--benchmark N`): step i feeds token t_i at position pos0+i and
 * t_{i+1} = argmax of its logits, t_0 = first_token. tokens_host[n_steps] receives t_1..t_n.
 * last_logits_host (nullable) receives the logits of the final step. */
q3_status q3_decode_greedy(q3_model* model, int32_t first_token, int pos0, int n_steps,
                           int32_t* tokens_host, float* last_logits_host);

/* Teacher-forced decode: feeds tokens_host[i] at position pos0+i for i < n and writes the
 * greedy argmax of every step to argmax_host[n] (nullable) and all logits to
 * logits_host[n*vocab] (nullable). */
q3_status q3_decode_forced(q3_model* model, const int32_t* tokens_host, int n, int pos0,
                           int32_t* argmax_host, float* logits_host);

/* Qwen3::Generate on token IDs (src/inference.cpp:639-700 without the tokenizer): prefill of
 * the prompt (empty prompt -> [bos]), then greedy tokens until max_new_tokens or, when
 * stop_on_eos, the EOS id. out_tokens_host needs max_new_tokens entries. */
q3_status q3_generate(q3_model* model, const int32_t* prompt_host, int n_prompt,
                      size_t max_new_tokens, int stop_on_eos, int32_t* out_tokens_host,
                      size_t* n_out, q3_generation_stats* stats);

/* Model-owned CUDA stream (cudaStream_t) for callers that order their own work against it. */
q3_status q3_model_stream(q3_model* model, void** stream);

/* Decode paths (no reference counterpart: the reference has one CPU path). FUSED is one
 * persistent kernel per call that runs whole decode steps (Qwen3-0.6B shape only); LAYERWISE is
 * a CUDA graph of per-layer kernels (any shape). Both run on the GPU; FUSED is the default when
 * the model's shape allows it. */
enum { Q3_PATH_LAYERWISE = 0, Q3_PATH_FUSED = 1 };
q3_status q3_model_set_decode_path(q3_model* model, int path);
q3_status q3_model_decode_path(const q3_model* model, int* path);
/* Failure-path check of the fused kernel's bounded waits: runs one launch whose grid-wide wait
 * can never be satisfied, with a ~10 ms bound, and reports in *timed_out whether the kernel
 * returned with its timeout status set. The model stays usable afterwards. */
q3_status q3_model_fused_timeout_selftest(q3_model* model, int* timed_out);
/* Instrumentation of the fused kernel (no reference counterpart): runs one decode step of
 * `token` at `pos` and writes globaltimer nanosecond stamps [n_phases][grid][8] (0 phase entry,
 * 1 phase start, 2-5 points inside the phase, 6 work done, 7 arrival; unset stamps are 0) to
 * stamps_host (capacity in elements). */
q3_status q3_model_fused_profile(q3_model* model, int32_t token, int pos, uint64_t* stamps_host,
                                 size_t capacity, int* n_phases, int* grid);

/* ------------------------------------------------------------------ batched decode
 * Independent sequences decoded together on one GPU (the data-parallel serving configuration).
 * The reference runs one sequence at a time (Qwen3::Generate, src/inference.cpp:639-700); a
 * batch produces, for every sequence, the tokens that Generate's greedy loop would (prefill of
 * the prompt, then one greedy token per step, no EOS stop), with every decode step of all
 * sequences computed at once: the weights are read once per step for all of them. The batch owns
 * a paged KV pool (16-token pages, a contiguous page range per sequence) sized for max_seqs
 * sequences of up to max_tokens positions (prompt + generated); positions never wrap. The model
 * handle must outlive the batch; the model's own single-sequence state is not touched. */
typedef struct q3_batch q3_batch;
q3_status q3_batch_create(q3_model* model, int max_seqs, int max_tokens, q3_batch** out);
void q3_batch_free(q3_batch* batch);
/* Adds a sequence and prefills its prompt (batched, on the tensor cores): *slot (nullable)
 * receives its index, *next_token_host (nullable) the greedy token after the prompt,
 * last_logits_host (nullable, vocab_size floats) the prompt's last logits. */
q3_status q3_batch_add(q3_batch* batch, const int32_t* ids_host, int n, int* slot,
                       int32_t* next_token_host, float* last_logits_host);
/* Adds n_seqs sequences at once: prompt i is the next lens_host[i] tokens of ids_host (the
 * prompts back to back). Prompts of up to 4096 tokens are prefilled together, one tensor-core
 * pass over the tokens of all of them per 4096-token chunk, each token's K/V written into its own
 * sequence's pages (the data-parallel configuration's many prompts); longer prompts are
 * prefilled one by one. *first_slot receives the slot of the first (the others follow);
 * next_tokens_host[n_seqs] and last_logits_host[n_seqs][vocab] (both nullable) as
 * q3_batch_add's. (The reference prefills one sequence, token by token:
 * src/inference.cpp:669-671.) */
q3_status q3_batch_add_many(q3_batch* batch, const int32_t* ids_host, const int* lens_host,
                            int n_seqs, int* first_slot, int32_t* next_tokens_host,
                            float* last_logits_host);
q3_status q3_batch_size(const q3_batch* batch, int* n_seqs);
/* The batch's CUDA stream (cudaStream_t) for callers that order or time work against it. */
q3_status q3_batch_stream(q3_batch* batch, void** stream);
/* n_steps greedy decode steps for every sequence; tokens_host[n_steps][n_seqs] (nullable)
 * receives the generated tokens (step-major). */
q3_status q3_batch_decode(q3_batch* batch, int n_steps, int32_t* tokens_host);
/* Teacher-forced steps: feeds tokens_host[step][n_seqs]; argmax_host[n_steps][n_seqs] receives
 * each step's greedy argmax, logits_host[n_steps][n_seqs][vocab_size] (nullable) all logits. */
q3_status q3_batch_decode_forced(q3_batch* batch, const int32_t* tokens_host, int n_steps,
                                 int32_t* argmax_host, float* logits_host);
/* Row `pos` of sequence `slot`'s layer-`layer` K/V (n_kv_heads*head_dim values each). */
q3_status q3_batch_kv_row(q3_batch* batch, int slot, int layer, int pos, uint16_t* k_host,
                          uint16_t* v_host);

/* ------------------------------------------------------------------ tensor-parallel decode
 * Single-sequence greedy decode split over the GPUs of one node, one process (and model handle)
 * per GPU (no reference counterpart: the reference runs on one CPU). Rank r of `world` computes
 * query heads [r*16/world, ...), KV heads [r*8/world, ...), MLP rows/columns
 * [r*H/world, ...) and a slice of the vocabulary; after o_proj and down_proj the ranks all-reduce
 * their partial sums over NVLink peer memory (a kernel of this library, not NCCL), and the argmax
 * likewise. Every rank prefills the prompt on its own model first (q3_prefill, full width), so
 * that the KV cache of its local heads is in place. world must divide the KV heads (1, 2, 4, 8).
 * Setup: q3_tp_create on every rank, exchange the 64-byte handles of q3_tp_ipc_handle (any
 * host channel), q3_tp_connect with all handles in rank order; then every rank calls the same
 * decode functions with the same arguments. */
typedef struct q3_tp q3_tp;
q3_status q3_tp_create(q3_model* model, int rank, int world, q3_tp** out);
void q3_tp_free(q3_tp* tp);
q3_status q3_tp_ipc_handle(q3_tp* tp, void* handle_host);
q3_status q3_tp_connect(q3_tp* tp, const void* handles_host);
q3_status q3_tp_stream(q3_tp* tp, void** stream);
/* n_steps greedy steps from first_token at position pos0 (positions < pos0 already in the cache);
 * tokens_host[n_steps] (nullable) receives the generated tokens, identical on every rank. */
q3_status q3_tp_decode(q3_tp* tp, int32_t first_token, int pos0, int n_steps,
                       int32_t* tokens_host);
/* Teacher-forced: feeds tokens_host[i] at pos0 + i; argmax_host[n] receives each step's argmax. */
q3_status q3_tp_decode_forced(q3_tp* tp, const int32_t* tokens_host, int n, int pos0,
                              int32_t* argmax_host);
/* solo_allreduce != 0: at world 1, the o_proj / down_proj partials go through the all-reduce
 * kernel with this rank as its only member (default: added into the residual directly).
 * wait_cycles: budget in SM clock cycles of every bounded flag wait (default 4e9, ~2 s). Every
 * rank of a group configures alike. A wait that runs out makes decode return
 * Q3_ERR_DEVICE_TIMEOUT; the decoder then refuses to decode (Q3_ERR_RUNTIME) until
 * q3_tp_reset, which every rank calls (and the ranks meet on the host) before decoding again. */
q3_status q3_tp_configure(q3_tp* tp, int solo_allreduce, long long wait_cycles);
q3_status q3_tp_reset(q3_tp* tp);
/* How the steps run (every rank of a group alike): Q3_TP_FUSED, the default where the model has
 * the fused decode kernel, is one persistent kernel per GPU for up to 256 steps that sends its
 * o_proj partials, down-projection sums and greedy candidates to every rank from inside its
 * phases (with solo_allreduce at world 1 they go through this rank's own exchange words);
 * Q3_TP_GRAPH is one CUDA graph per step with this library's all-reduce kernels;
 * Q3_TP_GRAPH_NCCL, a comparison arm, is the same graph with ncclAllReduce / ncclAllGather
 * captured in their place (needs q3_tp_nccl_connect; NCCL is loaded at run time). */
enum { Q3_TP_FUSED = 0, Q3_TP_GRAPH = 1, Q3_TP_GRAPH_NCCL = 2 };
q3_status q3_tp_set_path(q3_tp* tp, int path);
q3_status q3_tp_path(q3_tp* tp, int* path);
/* NCCL communicator of Q3_TP_GRAPH_NCCL: one process makes a 128-byte unique id, every rank
 * connects with the same id. */
q3_status q3_tp_nccl_unique_id(void* id_host);
q3_status q3_tp_nccl_connect(q3_tp* tp, const void* id_host);

/* ------------------------------------------------------------------ one block (class Block) */

/* Block(config, weights) (src/inference.cpp:720-730) with BlockWeights
 * (include/inference.h:163-176) given as 11 host arrays of bf16 bits in the order attn_norm,
 * q_norm, k_norm, wq, wk, wv, wo, mlp_norm, w1, w2, w3; sizes are checked as
 * Block::ValidateWeights does (src/inference.cpp:737-764) against the element counts given in
 * `counts` (nullable: then sizes are taken as valid). The cache holds cfg->max_seq_len rows. */
q3_status q3_block_create(const q3_config* cfg, const uint16_t* const* weights_host,
                          const size_t* counts, int device, q3_block** out);
void q3_block_free(q3_block* block);

/* Block::forward (src/inference.cpp:766-866) on a host vector x_host[dim], in place. */
q3_status q3_block_forward(q3_block* block, float* x_host, int pos, int num_sink, int kv_pos,
                           int kv_len);
/* Block::ResetCache (src/inference.cpp:732-735). */
q3_status q3_block_reset_cache(q3_block* block);
/* Block::GetCache (include/inference.h:193-195), reference layout [max_seq_len, kv_dim]. */
q3_status q3_block_get_cache(q3_block* block, uint16_t* k_host, uint16_t* v_host);
/* Fills the cache from the reference layout (the block test writes it through a const_cast). */
q3_status q3_block_set_cache(q3_block* block, const uint16_t* k_host, const uint16_t* v_host);

/* ------------------------------------------------------------------ free kernels (device ptrs)
 * The free functions of include/inference.h:308-315 and Sampler::Greedy (:204-207), on device
 * pointers, enqueued on `stream` (a cudaStream_t; NULL = legacy default stream). They return
 * after enqueueing. */

/* RmsNorm (src/inference.cpp:887-923). out may alias x. */
q3_status q3_rmsnorm(float* out, const float* x, const uint16_t* w, float eps, int n,
                     void* stream);
/* Softmax (src/inference.cpp:925-946). out may alias x. */
q3_status q3_softmax(float* out, const float* x, int n, void* stream);
/* MatMul (src/inference.cpp:952-966): out[n] = W[n,m] . x[m], W bf16 row-major. */
q3_status q3_matmul(float* out, const float* x, const uint16_t* w, int n, int m, void* stream);
/* ApplyRotaryEmb (src/inference.cpp:968-991), in place on x[d]. cos/sin are evaluated on the
 * host with the reference's fp32 expressions and passed to the kernel. */
q3_status q3_rope(float* x, int d, int head_dim, int pos, float theta, int rotary_dim,
                  void* stream);
/* FeedForwardNetwork (src/inference.cpp:993-1015). lin1/lin2 are [hidden_dim] scratch. */
q3_status q3_ffn(float* out, float* lin1, float* lin2, const float* x, const uint16_t* w1,
                 const uint16_t* w2, const uint16_t* w3, int hidden_dim, int dim, void* stream);

/* FastAttn (src/inference.cpp:1017-1058) for ONE query head over a bf16 cache in the reference
 * layout: k/v point at the head's first element, rows are n_kv_heads*head_dim apart. The
 * reference's `atth` scores buffer becomes `workspace`, whose size in bytes is
 * q3_attn_workspace_size(head_dim, kv_len); it holds the split-K partial results. */
size_t q3_attn_workspace_size(int head_dim, int kv_len);
q3_status q3_attn(float* out, void* workspace, const float* q, const uint16_t* k,
                  const uint16_t* v, int head_dim, int n_kv_heads, int kv_len, void* stream);

/* q3_attn without a workspace, for callers that cannot allocate device memory when they call in
 * (runtimes that own a fixed, pre-planned device-memory budget; callers that must avoid the device
 * synchronisation cudaMalloc/cudaFree can cause). No counterpart in the reference, which runs on
 * the CPU with caller-provided buffers. The split-K scratch is a static device array of
 * q3_attn_noalloc_max_scratch() bytes (66,304: 64 splits of head_dim up to 256), held by every GPU
 * that loads the library until exit; sizes that would need more are rejected with
 * Q3_ERR_INVALID_ARGUMENT. The first call on each device looks up the array's device address with
 * that device current - make it before any stream capture. All calls on a device share the
 * array: calls that may overlap on the GPU race and must be ordered by the caller. Nothing in the
 * array needs clearing between calls. Allocates nothing. */
size_t q3_attn_noalloc_max_scratch(void);
q3_status q3_attn_noalloc(float* out, const float* q, const uint16_t* k, const uint16_t* v,
                          int head_dim, int n_kv_heads, int kv_len, void* stream);

/* Tensor-core contraction used by the batched prefill (no reference counterpart; the reference's
 * MatMul is one fp32 vector at a time): out[M, N] = epilogue(A[M, K] . W[N, K]^T) with A and W bf16
 * row-major, fp32 accumulation. epilogue Q3_GEMM_STORE_F32 writes fp32 out[M, N];
 * Q3_GEMM_ADD_F32 adds into fp32 out[M, N]; Q3_GEMM_STORE_BF16 writes bf16 out[M, N];
 * Q3_GEMM_SWIGLU writes bf16 out[M, N] = silu(A . W^T) * (A . W3^T) (W and W3 both [N, K]).
 * K must be a multiple of 64; N a multiple of 128; all pointers 16-byte aligned. Synchronises
 * `stream` and reports a device timeout of the pipeline as Q3_ERR_DEVICE_TIMEOUT. */
enum { Q3_GEMM_STORE_F32 = 0, Q3_GEMM_ADD_F32 = 1, Q3_GEMM_SWIGLU = 2, Q3_GEMM_STORE_BF16 = 3 };
q3_status q3_gemm_bf16(void* out, const uint16_t* a, const uint16_t* w, const uint16_t* w3, int M,
                       int N, int K, int epilogue, void* stream);
/* As q3_gemm_bf16 with fp16 A and W (and W3); Q3_GEMM_SWIGLU and Q3_GEMM_STORE_BF16 then write
 * fp16 (saturated to +-65504). The operand precision of the default batched prefill. */
q3_status q3_gemm_f16(void* out, const uint16_t* a, const uint16_t* w, const uint16_t* w3, int M,
                      int N, int K, int epilogue, void* stream);

/* Sampler::Greedy (src/inference.cpp:703-709): index of the first maximum of logits[n], written
 * to *out_index (device int32). n == 0 is rejected like the reference's empty span. */
q3_status q3_greedy(const float* logits, int n, int32_t* out_index, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* Q3_B200_H */
