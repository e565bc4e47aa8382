/* abi_offsets.c - prints sizeof/offsetof of every structure the provider
   shares with the engine. TEST INFRASTRUCTURE: compiled once against the
   engine's own headers (backend/include/compute_backend.h,
   backend/core/llm_internal.h) to produce tests/golden/abi_offsets_ref.txt,
   and once against include/fyodor_b200_abi.h (-DFYB_MIRROR) by the tests;
   the two outputs must be identical. */
#ifdef FYB_MIRROR
#include "fyodor_b200_abi.h"
#else
#include "compute_backend.h"
#include "llm_internal.h"
#endif
#include <stddef.h>
#include <stdio.h>

#define S(T) printf("sizeof %s %zu\n", #T, sizeof(T));
#define F(T, f) printf("offsetof %s.%s %zu\n", #T, #f, offsetof(T, f));

int main(void)
{
    S(nya_compute_stats) F(nya_compute_stats, prefill_batch) F(nya_compute_stats, kernel_launches)
    F(nya_compute_stats, graph_replays) F(nya_compute_stats, external_matmul_kind) F(nya_compute_stats, tiled_attention_calls)
    S(nya_compute_attention) F(nya_compute_attention, batch) F(nya_compute_attention, scale)
    S(nya_backend_interface) F(nya_backend_interface, name) F(nya_backend_interface, capabilities)
    F(nya_backend_interface, create) F(nya_backend_interface, matvec) F(nya_backend_interface, plan_create)
    F(nya_backend_interface, plan_token) F(nya_backend_interface, plan_prefill) F(nya_backend_interface, plan_stats)
    F(nya_backend_interface, matmul) F(nya_backend_interface, attention_f32) F(nya_backend_interface, plan_read_kv)
    F(nya_backend_interface, context_stats)
    S(nya_llm_tensor) F(nya_llm_tensor, type) F(nya_llm_tensor, dimensions) F(nya_llm_tensor, data) F(nya_llm_tensor, data_size)
    S(nya_llm_layer) F(nya_llm_layer, feed_forward_up) F(nya_llm_layer, rope_factors) F(nya_llm_layer, head_count)
    F(nya_llm_layer, kv_source) F(nya_llm_layer, cache_offset)
    S(nya_llm_tokenizer) F(nya_llm_tokenizer, vocabulary_size) F(nya_llm_tokenizer, suppressed_tokens)
    F(nya_llm_tokenizer, suppressed_count)
    S(nya_llm_projector)
    S(nya_llm_context) F(nya_llm_context, tensors) F(nya_llm_context, tensor_count) F(nya_llm_context, layers)
    F(nya_llm_context, tokenizer) F(nya_llm_context, token_embedding) F(nya_llm_context, output_norm)
    F(nya_llm_context, output) F(nya_llm_context, embedding_length) F(nya_llm_context, block_count)
    F(nya_llm_context, context_length) F(nya_llm_context, norm_epsilon) F(nya_llm_context, rope_frequency_base)
    F(nya_llm_context, is_gemma) F(nya_llm_context, is_assistant) F(nya_llm_context, expert_count)
    F(nya_llm_context, final_logit_softcap) F(nya_llm_context, cache_width) F(nya_llm_context, maximum_query_length)
    F(nya_llm_context, maximum_hidden_length) F(nya_llm_context, layer_heads) F(nya_llm_context, sliding_rope_dimension)
    return 0;
}
