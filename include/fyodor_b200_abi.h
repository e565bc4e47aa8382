/* fyodor_b200_abi.h - the Fyodor engine's provider ABI, restated.
 *
 * These are the types the Fyodor C engine passes across its accelerator
 * provider boundary. The layouts must stay byte-identical to the engine's
 * own headers, because the engine hands these structures to the provider
 * by pointer:
 *   - nya_backend_type, capability bits, nya_compute_stats,
 *     nya_compute_attention        : backend/include/compute.h:9-34
 *   - nya_backend_interface        : backend/include/compute_backend.h:12-29
 *   - nya_llm_tensor / _layer / _tokenizer / _mapping / _projector /
 *     nya_llm_context              : backend/core/llm_internal.h:22-164
 * A test compiles an offsetof() dump of both definitions and compares them
 * (tests/test_abi_layout.py), so a drift in either side is caught on CPU.
 *
 * A build that already includes the engine's compute_backend.h and
 * llm_internal.h defines FYB_USE_ENGINE_HEADERS and skips this restatement.
 */
#ifndef FYODOR_B200_ABI_H
#define FYODOR_B200_ABI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef FYB_USE_ENGINE_HEADERS

/* ---- compute.h:7-34 ---------------------------------------------------- */
typedef struct nya_compute_context nya_compute_context;
typedef enum nya_backend_type {
    NYA_BACKEND_CPU, NYA_BACKEND_CUDA, NYA_BACKEND_VULKAN, NYA_BACKEND_ROCM, NYA_BACKEND_MLX
} nya_backend_type;
enum { NYA_COMPUTE_MATVEC = 1U, NYA_COMPUTE_QUANTIZED = 2U, NYA_COMPUTE_RESIDENT = 4U,
       NYA_COMPUTE_MATMUL = 8U };

typedef struct nya_compute_stats {
    size_t weights_bytes, kv_bytes, scratch_bytes, prefill_batch;
    size_t external_matmul_bytes;
    unsigned long long kernel_launches, uploads, downloads, synchronizations;
    unsigned long long external_matmul_calls;
    unsigned long long graph_captures, graph_replays;
    unsigned external_matmul_kind;
    unsigned long long cutlass_matmul_calls;
    unsigned long long tiled_attention_calls;
} nya_compute_stats;

typedef struct nya_compute_attention {
    const float *query, *keys, *values;
    float *output;
    size_t batch, heads, kv_heads, width, capacity, position, window;
    float scale;
} nya_compute_attention;

/* ---- compute_backend.h:11-29 -------------------------------------------- */
struct nya_llm_context;
typedef struct nya_backend_interface {
    nya_backend_type type;
    const char *name;
    unsigned capabilities;
    void *(*create)(void);
    void (*destroy)(void *);
    int (*active)(const void *);
    int (*matvec)(void *, const void *, size_t, size_t, unsigned, const float *, float *);
    void *(*plan_create)(void *, const struct nya_llm_context *, size_t);
    void (*plan_free)(void *);
    int (*plan_token)(void *, uint32_t, size_t, int, float *);
    int (*plan_prefill)(void *, const uint32_t *, size_t, size_t, float *);
    void (*plan_stats)(const void *, nya_compute_stats *);
    int (*matmul)(void *, const void *, size_t, size_t, unsigned, const float *, float *, size_t);
    int (*attention_f32)(void *, const nya_compute_attention *);
    int (*plan_read_kv)(void *, size_t, size_t, size_t, float *, float *, size_t);
    void (*context_stats)(const void *, nya_compute_stats *);
} nya_backend_interface;

/* ---- llm_internal.h:11-164 ---------------------------------------------- */
enum nya_llm_tensor_type {
    NYA_LLM_TENSOR_F32 = 0,
    NYA_LLM_TENSOR_F16 = 1,
    NYA_LLM_TENSOR_Q4_0 = 2,
    NYA_LLM_TENSOR_Q8_0 = 8,
    NYA_LLM_TENSOR_Q4_K = 12,
    NYA_LLM_TENSOR_Q6_K = 14,
    NYA_LLM_TENSOR_BF16 = 30
};

/* dimensions[0] = columns (inputs), dimensions[1] = rows (outputs). */
typedef struct nya_llm_tensor {
    char name[128];
    uint32_t type;
    uint32_t dimension_count;
    uint64_t dimensions[4];
    uint64_t relative_offset;
    const unsigned char *data;
    size_t data_size;
    int bound;
} nya_llm_tensor;

typedef struct nya_llm_layer {
    const nya_llm_tensor *attention_norm;
    const nya_llm_tensor *query;
    const nya_llm_tensor *key;
    const nya_llm_tensor *value;
    const nya_llm_tensor *attention_output;
    const nya_llm_tensor *feed_forward_norm;
    const nya_llm_tensor *feed_forward_gate;
    const nya_llm_tensor *feed_forward_down;
    const nya_llm_tensor *feed_forward_up;
    const nya_llm_tensor *query_norm, *key_norm, *attention_post_norm, *ffn_post_norm;
    const nya_llm_tensor *router, *router_scale, *expert_scale;
    const nya_llm_tensor *expert_gate, *expert_up, *expert_gate_up, *expert_down;
    const nya_llm_tensor *expert_pre_norm, *shared_post_norm, *expert_post_norm;
    const nya_llm_tensor *ple_gate, *ple_projection, *ple_norm, *output_scale;
    const nya_llm_tensor *rope_factors;
    uint32_t head_count, kv_head_count, head_dimension, hidden_length;
    uint32_t expert_hidden_length, sliding_window, kv_source;
    /* KV offsets count float elements per sequence position. */
    size_t cache_offset;
} nya_llm_layer;

typedef struct nya_llm_token_index {
    const char *piece;
    uint32_t token;
} nya_llm_token_index;

typedef struct nya_llm_bpe_rule {
    char *text;
    size_t left_length;
    uint32_t rank;
} nya_llm_bpe_rule;

typedef struct nya_llm_tokenizer {
    char **pieces;
    size_t *piece_lengths;
    float *scores;
    int32_t *types;
    nya_llm_token_index *sorted;
    uint32_t vocabulary_size;
    size_t maximum_piece_length;
    int32_t byte_tokens[256];
    uint32_t unknown_token;
    uint32_t beginning_token;
    uint32_t end_token;
    int add_beginning_token;
    int add_end_token;
    int add_space_prefix;
    int uses_sentencepiece_space;
    int uses_merge_ranks;
    nya_llm_bpe_rule *merges;
    size_t merge_count;
    unsigned char *stop_tokens;
    uint32_t *suppressed_tokens;
    size_t suppressed_count;
    uint32_t *special_tokens;
    size_t special_count;
} nya_llm_tokenizer;

typedef struct nya_llm_mapping {
    unsigned char *data;
    size_t size;
    uintptr_t file_handle;
    uintptr_t mapping_handle;
} nya_llm_mapping;

typedef struct nya_llm_projector {
    char vision_type[32], audio_type[32];
    uint32_t vision_width, audio_width, output_width, audio_output_width;
    uint32_t vision_blocks, audio_blocks, patch_size, position_count;
    float vision_epsilon, audio_epsilon;
    const nya_llm_tensor *patch, *patch_bias, *position, *vision, *audio;
    const nya_llm_tensor *norm_weight[3], *norm_bias[3];
} nya_llm_projector;

typedef struct nya_llm_context {
    nya_compute_context *compute;
    nya_llm_mapping mapping;
    size_t metadata_end;
    size_t file_type_begin, file_type_end;
    uint64_t gguf_metadata_count;
    uint32_t tensor_alignment;
    nya_llm_tensor *tensors;
    size_t tensor_count;
    nya_llm_layer *layers;
    nya_llm_tokenizer tokenizer;
    nya_llm_projector projector;
    const nya_llm_tensor *token_embedding;
    const nya_llm_tensor *output_norm;
    const nya_llm_tensor *output;
    uint32_t embedding_length;
    uint32_t feed_forward_length;
    uint32_t block_count;
    uint32_t head_count;
    uint32_t key_value_head_count;
    uint32_t context_length;
    uint32_t rope_dimension_count;
    float norm_epsilon;
    float rope_frequency_base;
    int is_gemma;
    int is_assistant;
    uint32_t backbone_length, nextn_layers;
    const nya_llm_tensor *nextn_pre, *nextn_post;
    uint32_t head_dimension, sliding_head_dimension, sliding_window, shared_kv_layers;
    uint32_t per_layer_embedding_length, expert_count, experts_used;
    float sliding_rope_base, final_logit_softcap;
    const nya_llm_tensor *ple_embedding, *ple_projection, *ple_norm;
    size_t cache_width, maximum_query_length, maximum_hidden_length;
    uint32_t layer_heads[256], layer_kv_heads[256], layer_hidden[256];
    uint32_t layer_expert_hidden[256], layer_sliding[256];
    uint32_t heads_count, kv_heads_count, hidden_count, expert_hidden_count, sliding_count;
    uint32_t value_dimension, sliding_value_dimension, sliding_rope_dimension;
} nya_llm_context;

#endif /* FYB_USE_ENGINE_HEADERS */

#ifdef __cplusplus
}
#endif
#endif
