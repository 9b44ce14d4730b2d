// gpt_sovits::t2s_* -- the T2S model/session interface of GPT-SoVITS.cpp
// (include/gpt_sovits/t2s.h of the reference), served by the B200 library libt2sx.so.
//
// Same names, signatures, struct fields and call sequence as the reference's session-level API
// (t2s.h:215-582): t2s_model_load(fname, model, backend), t2s_session_init(session, hparams,
// backend, n_batch, slot_size, sampler_cfg, kv_cache_type), the flex-plan prefill, the persistent
// decode graph and their tensor accessors.  A caller drives it exactly as the reference's decode
// loop does (tests/t2s/test_t2s_infer.cpp:204-421): ggml_backend_tensor_set on the input
// tensors, t2s_session_decode_advance / t2s_session_flex_advance, ggml_backend_graph_compute,
// ggml_backend_tensor_get on the outputs.  The ggml types come from the minimal shim headers next
// to this one (ggml.h, ggml-backend.h, ggml-cuda.h); the backend is a CUDA device
// (ggml_backend_cuda_init).  Differences from the reference, all checked on the host:
//   * the KV cache is f16 and paged on the device: kv_cache_type must be GGML_TYPE_F16
//     (t2s_session_init returns false for any other type);
//   * the ggml graph builders (t2s_attention_block_forward, t2s_sampler_block_forward,
//     t2s_embed_*_forward) are not provided -- they take a ggml_context and only make sense
//     inside ggml; t2s_session_embed_input builds the prefill rows instead;
//   * KV caches, masks and weights are read-only views (tensor_get works, tensor_set aborts);
//   * exp_noise is used once set (the stochastic chain); until then sampled == greedy;
//   * prefill rows sample with an empty seen set (the reference's tests pass zeros there);
//   * t2s_sampler_config has one more field, eos_mask (default false): logit[eos] is masked,
//     for fixed-length decoding.
// Errors follow the reference: load / init / build return false (or an empty graph) and print
// to stderr; illegal slot transitions abort through GGML_ASSERT.  Free functions are idempotent.
#pragma once

#include "../ggml.h"
#include "../ggml-alloc.h"
#include "../ggml-backend.h"

#include <cstdint>
#include <string>
#include <vector>

#if defined(__GNUC__)
#define GPT_SOVITS_API __attribute__((visibility("default")))
#else
#define GPT_SOVITS_API
#endif

struct t2sx_model;

namespace gpt_sovits {

// ---- weights (t2s.h:56-169): shapes and types of the GGUF tensors; the data lives repacked on
// the device, so these tensors carry no host data ----
struct sovits_extract_latent_block_weights {
    struct ggml_tensor* ssl_proj_w;   // {2, 768, 768}
    struct ggml_tensor* ssl_proj_b;   // {768}
    struct ggml_tensor* codebook;     // {768, 1024}
};

struct t2s_embed_block_weights {
    struct ggml_tensor* text_embedding;    // {d_model, phoneme_vocab}
    struct ggml_tensor* bert_proj_w;       // {1024, d_model}
    struct ggml_tensor* bert_proj_b;       // {d_model}
    struct ggml_tensor* text_pos_alpha;    // {1}
    struct ggml_tensor* audio_embedding;   // {d_model, semantic_vocab}
    struct ggml_tensor* audio_pos_alpha;   // {1}
};

struct t2s_attention_block_weights {
    struct ggml_tensor* qkv_w;        // {d_model, 3*d_model}
    struct ggml_tensor* qkv_b;        // {3*d_model}
    struct ggml_tensor* out_proj_w;   // {d_model, d_model}
    struct ggml_tensor* out_proj_b;   // {d_model}
    struct ggml_tensor* ln1_w;        // {d_model}
    struct ggml_tensor* ln1_b;        // {d_model}
    struct ggml_tensor* ffn_up_w;     // {d_model, d_ff}
    struct ggml_tensor* ffn_up_b;     // {d_ff}
    struct ggml_tensor* ffn_down_w;   // {d_ff, d_model}
    struct ggml_tensor* ffn_down_b;   // {d_model}
    struct ggml_tensor* ln2_w;        // {d_model}
    struct ggml_tensor* ln2_b;        // {d_model}
};

// ---- model (t2s.h:215-272) ----
struct t2s_hparams {
    uint32_t embedding_dim      = 512;
    uint32_t hidden_dim         = 512;
    uint32_t n_head             = 16;
    uint32_t linear_units       = 2048;
    uint32_t n_layer            = 24;
    uint32_t vocab_size         = 1025;
    uint32_t phoneme_vocab_size = 732;
    uint32_t eos                = 1024;
    uint32_t inter_channels     = 192;
};

struct t2s_model_weights {
    sovits_extract_latent_block_weights extract_latent;
    t2s_embed_block_weights embed;
    std::vector<t2s_attention_block_weights> attention;
    struct ggml_tensor* lm_head_w;   // {d_model, vocab}
};

struct t2s_model {
    t2s_hparams hparams = {};
    t2s_model_weights weights = {};
    ggml_backend_t backend = nullptr;         // borrowed
    ggml_backend_buffer_t buf_w = nullptr;    // owned (the device weights)
    struct ggml_context* ctx_w = nullptr;     // owned (the weight tensors' descriptions)
    t2sx_model* handle = nullptr;             // this implementation: the loaded model
};

// Loads the GGUF written by convert_t2s_to_gguf.py onto the backend's device (loader.cpp:140-228).
GPT_SOVITS_API bool t2s_model_load(const std::string& fname, t2s_model& model, ggml_backend_t backend);
GPT_SOVITS_API void t2s_model_free(t2s_model& model);

// ---- sampler configuration (t2s.h:279-284) ----
struct t2s_sampler_config {
    int   top_k              = 15;
    float top_p              = 1.0f;
    float temperature        = 1.0f;
    float repetition_penalty = 1.35f;
    bool  eos_mask           = false;   // this implementation: logit[eos] masked (fixed-length runs)
};

// ---- session (t2s.h:290-369) ----
struct t2s_session_impl;

struct t2s_session {
    uint32_t n_batch   = 0;
    uint32_t slot_size = 0;

    struct slot_state {
        int n_pos        = 0;
        int audio_offset = 0;
    };
    std::vector<slot_state> slots;

    std::vector<struct ggml_tensor*> k_caches;   // [n_layer] {d_model, n_batch*slot_size} F16 views
    std::vector<struct ggml_tensor*> v_caches;

    struct ggml_tensor* kv_pos = nullptr;   // {n_batch} I32
    struct ggml_tensor* mask   = nullptr;   // {n_batch*slot_size, n_batch} F16 view
    // Host mirror of the decode mask (mask_host[col * max_ctx + row]); kept while it has at most
    // 2^24 entries (n_batch^2 * slot_size), left empty above that -- read `mask` instead.
    std::vector<ggml_fp16_t> mask_host;

    enum ggml_type kv_cache_type = GGML_TYPE_F16;

    ggml_backend_t        backend = nullptr;   // borrowed
    ggml_backend_buffer_t buf_kv  = nullptr;   // owned (device KV pages)
    struct ggml_context*  ctx_kv  = nullptr;   // owned (the session's tensors)

    struct ggml_context* ctx_graph = nullptr;   // owned
    struct ggml_cgraph*  gf_dec    = nullptr;   // the decode step (t2s_session_build_decode_graph)
    ggml_gallocr_t       alloc_dec = nullptr;

    struct ggml_tensor* token_id = nullptr;   // {n_batch} I32 (caller fills)
    struct ggml_tensor* position = nullptr;   // {n_batch} I32 (decode_advance fills)
    struct ggml_tensor* pe_table = nullptr;   // {d_model, slot_size} F32

    t2s_sampler_config sampler_cfg;

    struct ggml_tensor* seen_mask = nullptr;   // {vocab, n_batch} F32 (caller fills)
    struct ggml_tensor* exp_noise = nullptr;   // {vocab, n_batch} F32 (caller fills)
    struct ggml_tensor* sampled   = nullptr;   // {n_batch} I32
    struct ggml_tensor* greedy    = nullptr;   // {n_batch} I32

    struct ggml_context*  ctx_ref       = nullptr;
    ggml_backend_buffer_t buf_ref       = nullptr;
    struct ggml_tensor*   ref_text_emb  = nullptr;   // {d_model, T_ref}
    struct ggml_tensor*   ref_audio_emb = nullptr;   // {d_model, T_prompt}
    int64_t               ref_T_ref     = 0;
    int64_t               ref_T_prompt  = 0;

    ggml_gallocr_t alloc_flex = nullptr;

    t2s_session_impl* impl = nullptr;   // this implementation: device session and host buffers
};

GPT_SOVITS_API bool t2s_session_init(t2s_session& session, const t2s_hparams& hparams, ggml_backend_t backend,
                                     uint32_t n_batch, uint32_t slot_size, const t2s_sampler_config& sampler_cfg = {},
                                     enum ggml_type kv_cache_type = GGML_TYPE_F32);
GPT_SOVITS_API void t2s_session_free(t2s_session& session);
GPT_SOVITS_API int t2s_session_find_free_slot(const t2s_session& session);
GPT_SOVITS_API void t2s_session_slot_release(t2s_session& session, int slot_id);
GPT_SOVITS_API void t2s_session_decode_advance(t2s_session& session);
GPT_SOVITS_API int t2s_session_slot_n_pos(const t2s_session& session, int slot_id);

struct t2s_layer_caches {
    struct ggml_tensor* k;
    struct ggml_tensor* v;
};

GPT_SOVITS_API t2s_layer_caches t2s_session_get_layer_caches(const t2s_session& session, int layer);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_kv_pos(const t2s_session& session);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_mask(const t2s_session& session);
GPT_SOVITS_API int t2s_session_get_n_kv(const t2s_session& session);

// Reference embedding (t2s.h:433-467): prompt codes from the HuBERT frames ({768, T_hub}) on the
// device, then the reference text rows (text embedding + BERT projection + positions 0..T_ref-1)
// and the prompt rows (code embedding + positions 0..T_prompt-1).
GPT_SOVITS_API bool t2s_session_compute_ref_emb(t2s_session& session, const t2s_model& model, const int32_t* ref_token,
                                                int64_t T_ref, const float* ref_bert, const float* hubert_data,
                                                int64_t T_hub);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_ref_text_emb(const t2s_session& session);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_ref_audio_emb(const t2s_session& session);
GPT_SOVITS_API int64_t t2s_session_get_ref_T_ref(const t2s_session& session);
GPT_SOVITS_API int64_t t2s_session_get_ref_T_prompt(const t2s_session& session);

// Persistent decode step (t2s.h:469-488): all n_batch slots must be decoding.
GPT_SOVITS_API bool t2s_session_build_decode_graph(t2s_session& session, const t2s_model& model);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_token_id(const t2s_session& session);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_position(const t2s_session& session);
GPT_SOVITS_API struct ggml_cgraph* t2s_session_get_decode_graph(const t2s_session& session);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_sampled(const t2s_session& session);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_greedy(const t2s_session& session);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_seen_mask(const t2s_session& session);
GPT_SOVITS_API struct ggml_tensor* t2s_session_get_exp_noise(const t2s_session& session);

// ---- flex plans: prefill and mixed prefill/decode steps (t2s.h:490-582) ----
struct t2s_batch_plan {
    std::vector<int> n_query;   // size n_batch; 0 idle, 1 decode, > 1 prefill
    int total() const {
        int t = 0;
        for (int q : n_query) t += q > 0 ? q : 0;
        return t;
    }
};

struct t2s_flex_graph {
    struct ggml_tensor* x_prefill        = nullptr;   // {d_model, N_prefill} F32 (caller fills)
    struct ggml_tensor* decode_token_ids = nullptr;   // {n_decode} I32 (caller fills)
    struct ggml_tensor* decode_positions = nullptr;   // {n_decode} I32 (flex_advance fills)
    struct ggml_tensor* kv_pos           = nullptr;   // {N} I32 (flex_advance fills)
    struct ggml_tensor* mask             = nullptr;   // {n_kv, N} F16 view
    struct ggml_tensor* y                = nullptr;   // {d_model, N} F32 final-layer rows
    struct ggml_tensor* seen_mask        = nullptr;   // {vocab, n_active} F32 (caller fills)
    struct ggml_tensor* exp_noise        = nullptr;   // {vocab, n_active} F32 (caller fills)
    struct ggml_tensor* sampled          = nullptr;   // {n_active} I32
    struct ggml_tensor* greedy           = nullptr;   // {n_active} I32
    struct ggml_context* ctx     = nullptr;   // non-null on success (owns the graph's state)
    struct ggml_cgraph*  gf      = nullptr;
    ggml_backend_t       backend = nullptr;   // borrowed from the session
    int N        = 0;
    int n_active = 0;
    int n_decode = 0;
};

GPT_SOVITS_API t2s_flex_graph t2s_session_build_flex_graph(t2s_session& session, const t2s_model& model,
                                                           const t2s_batch_plan& plan);
GPT_SOVITS_API void t2s_flex_graph_free(t2s_flex_graph& graph);
GPT_SOVITS_API void t2s_session_flex_advance(t2s_session& session, const t2s_batch_plan& plan, t2s_flex_graph& graph);

// ---- this implementation: prefill rows on the device (what the reference builds with its ggml
// graph builders, block.cpp:424-511) ----
// Rows f32 [T_text + T_prompt][d_model] of one prompt: text rows from phoneme ids and BERT
// features ({1024, T_text}) with positions from 0, then audio rows from semantic ids with
// positions from 0.
GPT_SOVITS_API bool t2s_session_embed_input(t2s_session& session, const t2s_model& model, const int32_t* phones,
                                            const float* bert, int64_t T_text, const int32_t* sem, int64_t T_prompt,
                                            float* x_out);
// The flex plan's prefill rows after t2s_session_compute_ref_emb: [reference text | input text |
// reference prompt], the input text's positions continuing after the reference text's; sets
// nothing in the session (ref_T_prompt is already the prompt length).
GPT_SOVITS_API bool t2s_session_build_prefill_input(t2s_session& session, const t2s_model& model,
                                                    const int32_t* input_token, int64_t T_in,
                                                    const float* input_bert, std::vector<float>& x_out);

}  // namespace gpt_sovits
