// C++ session-level T2S interface over libt2sx (include/t2sx.h), for hosts that drive the
// reference's gpt_sovits::t2s_* API (include/gpt_sovits/t2s.h of GPT-SoVITS.cpp).
//
// Same names, struct fields and call sequence as the reference's model / session / flex-plan /
// decode-graph functions (t2s.h:215-582), with the ggml handles replaced:
//   ggml_backend_t backend        -> int device (CUDA device index)
//   ggml tensors of the graphs    -> host vectors in the structs (x_prefill, decode_token_ids,
//                                    token_id, sampled, greedy)
//   ggml_backend_graph_compute    -> t2s_flex_graph_compute / t2s_session_decode_compute
// and the session binding the model at init (it runs on the model's device and weights), where the
// reference binds hparams + backend and passes the model at graph build.  The KV cache is f16,
// paged (the reference's kv_cache_type argument has no counterpart).
//
// Error behaviour follows the reference: load / init / build return false (or an empty graph)
// and print the reason to stderr; illegal slot transitions (prefill of an active slot, decode of
// an idle one, n_query < ref_T_prompt, running past slot_size, a bad slot id) abort with a message,
// as GGML_ASSERT does in session.cpp.  Free functions are idempotent.
//
// Flex plans: a plan may prefill idle slots and decode active ones in the same step.  The decode
// part runs on the persistent decode path, which steps every active slot, so a plan that decodes
// must give n_query = 1 to every active slot (leaving one idle in such a plan aborts); a
// prefill-only plan leaves the active slots untouched, as in the reference.
#ifndef GPT_SOVITS_T2S_CUDA_H
#define GPT_SOVITS_T2S_CUDA_H

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "../t2sx.h"

namespace gpt_sovits {

#define T2S_CUDA_ASSERT(cond, msg)                                                            \
    do {                                                                                      \
        if (!(cond)) {                                                                        \
            std::fprintf(stderr, "%s:%d: T2S_CUDA_ASSERT(%s) failed: %s\n", __FILE__, __LINE__, \
                         #cond, msg);                                                         \
            std::abort();                                                                     \
        }                                                                                     \
    } while (0)

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

struct t2s_model {
    t2s_hparams  hparams = {};
    int          device  = -1;       // replaces the borrowed ggml backend
    t2sx_model * handle  = nullptr;  // owned: weights on the device
};

inline bool t2s_model_load(const std::string & fname, t2s_model & model, int device = 0) {
    t2sx_model * h = nullptr;
    if (t2sx_model_load(fname.c_str(), device, &h) != T2SX_OK) {
        std::fprintf(stderr, "t2s_model_load: %s\n", t2sx_last_error());
        return false;
    }
    uint32_t hp[9];
    int32_t wt[4];
    t2sx_model_hparams(h, hp, wt);
    model.hparams = t2s_hparams{hp[0], hp[1], hp[2], hp[3], hp[4], hp[5], hp[6], hp[7], hp[8]};
    model.device = device;
    model.handle = h;
    return true;
}

inline void t2s_model_free(t2s_model & model) {
    if (model.handle) t2sx_model_free(model.handle);
    model.handle = nullptr;
    model.device = -1;
}

// ---- session (t2s.h:279-418) ----
struct t2s_sampler_config {
    int   top_k              = 15;
    float top_p              = 1.0f;
    float temperature        = 1.0f;
    float repetition_penalty = 1.35f;
};

struct t2s_session {
    uint32_t n_batch   = 0;
    uint32_t slot_size = 0;
    t2s_sampler_config sampler_cfg;
    int64_t ref_T_prompt = 0;        // prompt audio tokens of the session's reference (as in t2s.h)
    int64_t ref_T_ref = 0;           // reference text tokens
    std::vector<int32_t> ref_tokens, ref_codes;   // reference phonemes, prompt codes (from HuBERT)
    std::vector<float> ref_bert;                  // reference BERT features [T_ref][1024]
    // persistent decode path (t2s.h:477-488): caller fills token_id, reads sampled / greedy
    std::vector<int32_t> token_id;   // {n_batch}, slot order
    std::vector<int32_t> sampled;    // {n_batch}
    std::vector<int32_t> greedy;     // {n_batch}
    bool decode_ready = false;
    bool advanced     = false;
    t2sx_session * handle = nullptr;  // owned
};

// The reference's t2s_session_init(session, hparams, backend, n_batch, slot_size, sampler_cfg,
// kv_cache_type); eos_mask masks EOS in the sampler (a harness rule of fixed-length runs).
inline bool t2s_session_init(t2s_session & session, const t2s_model & model, uint32_t n_batch, uint32_t slot_size,
                             const t2s_sampler_config & sampler_cfg = {}, bool eos_mask = false) {
    if (!model.handle) {
        std::fprintf(stderr, "t2s_session_init: model not loaded\n");
        return false;
    }
    t2sx_sampler_config c{sampler_cfg.top_k, sampler_cfg.top_p, sampler_cfg.temperature,
                          sampler_cfg.repetition_penalty, eos_mask ? 1 : 0};
    t2sx_session * h = nullptr;
    if (t2sx_session_create(model.handle, n_batch, slot_size, &c, &h) != T2SX_OK) {
        std::fprintf(stderr, "t2s_session_init: %s\n", t2sx_last_error());
        return false;
    }
    session.n_batch = n_batch;
    session.slot_size = slot_size;
    session.sampler_cfg = sampler_cfg;
    session.ref_T_prompt = 0;
    session.token_id.assign(n_batch, 0);
    session.sampled.assign(n_batch, 0);
    session.greedy.assign(n_batch, 0);
    session.decode_ready = false;
    session.advanced = false;
    session.handle = h;
    return true;
}

inline void t2s_session_free(t2s_session & session) {
    if (session.handle) t2sx_session_free(session.handle);
    session.handle = nullptr;
    session.decode_ready = false;
}

inline int t2s_session_find_free_slot(const t2s_session & session) { return t2sx_session_find_free_slot(session.handle); }

inline void t2s_session_slot_release(t2s_session & session, int slot_id) {
    T2S_CUDA_ASSERT(slot_id >= 0 && (uint32_t)slot_id < session.n_batch, "slot id out of range");
    T2S_CUDA_ASSERT(t2sx_session_slot_release(session.handle, slot_id) == T2SX_OK, t2sx_last_error());
}

inline int t2s_session_slot_n_pos(const t2s_session & session, int slot_id) {
    T2S_CUDA_ASSERT(slot_id >= 0 && (uint32_t)slot_id < session.n_batch, "slot id out of range");
    return t2sx_session_slot_n_pos(session.handle, slot_id);
}

// Total KV entries (t2s_session_get_n_kv, t2s.h:431): always n_batch * slot_size.
inline int t2s_session_get_n_kv(const t2s_session & session) { return (int)(session.n_batch * session.slot_size); }

// Prefill input rows of one prompt (t2s_embed_input_forward / t2s_embed_ref_forward,
// block.cpp:424-511): x_out f32 [T_text + T_prompt][d_model] (host).
inline bool t2s_embed_input(t2s_session & session, const int32_t * phones, const float * bert, int T_text,
                            const int32_t * sem, int T_prompt, float * x_out) {
    if (t2sx_embed_prefill(session.handle, phones, bert, T_text, sem, T_prompt, x_out, 0) != T2SX_OK) {
        std::fprintf(stderr, "t2s_embed_input: %s\n", t2sx_last_error());
        return false;
    }
    return true;
}

// ---- reference prompt (t2s.h:432-467) ----
// t2s_session_compute_ref_emb: the prompt semantic codes are extracted from the HuBERT frames
// ({768, T_hub} in ggml order = [T_hub][768]) on the device (Conv1d k=2 s=2 + nearest code), and
// the reference text is kept; t2s_embed_with_ref then builds the prefill rows
// [reference text | input text | reference prompt] and sets ref_T_prompt.
inline bool t2s_session_compute_ref_emb(t2s_session & session, const t2s_model & model, const int32_t * ref_token,
                                        int64_t T_ref, const float * ref_bert, const float * hubert_data, int64_t T_hub) {
    T2S_CUDA_ASSERT(session.handle != nullptr && model.handle != nullptr, "session or model not initialised");
    T2S_CUDA_ASSERT(ref_token != nullptr && ref_bert != nullptr && hubert_data != nullptr, "null input");
    T2S_CUDA_ASSERT(T_ref > 0 && T_hub > 0, "empty reference");
    if (T_hub < 2) {
        std::fprintf(stderr, "t2s_session_compute_ref_emb: at least 2 HuBERT frames are needed\n");
        return false;
    }
    std::vector<int32_t> codes((size_t)((T_hub - 2) / 2 + 1));
    if (t2sx_extract_latent(session.handle, hubert_data, (int32_t)T_hub, codes.data()) != T2SX_OK) {
        std::fprintf(stderr, "t2s_session_compute_ref_emb: %s\n", t2sx_last_error());
        return false;
    }
    session.ref_codes = std::move(codes);
    session.ref_tokens.assign(ref_token, ref_token + T_ref);
    session.ref_bert.assign(ref_bert, ref_bert + T_ref * 1024);
    session.ref_T_ref = T_ref;
    session.ref_T_prompt = (int64_t)session.ref_codes.size();
    return true;
}
inline int64_t t2s_session_get_ref_T_ref(const t2s_session & session) { return session.ref_T_ref; }
inline int64_t t2s_session_get_ref_T_prompt(const t2s_session & session) { return session.ref_T_prompt; }

// The reference's cached embeddings (t2s_session_get_ref_text_emb / get_ref_audio_emb,
// t2s.h:458-461) as host rows f32 [T][d_model]: the reference text rows (text embedding + BERT
// projection + positions 0..T_ref-1) and the prompt rows (code embedding + positions
// 0..T_prompt-1).  Empty before t2s_session_compute_ref_emb.
inline std::vector<float> t2s_session_get_ref_text_emb(t2s_session & session, const t2s_model & model) {
    if (session.ref_T_ref <= 0) return {};
    std::vector<float> x((size_t)(session.ref_T_ref + session.ref_T_prompt) * model.hparams.embedding_dim);
    if (!t2s_embed_input(session, session.ref_tokens.data(), session.ref_bert.data(), (int)session.ref_T_ref,
                         session.ref_codes.data(), (int)session.ref_T_prompt, x.data()))
        return {};
    x.resize((size_t)session.ref_T_ref * model.hparams.embedding_dim);
    return x;
}
inline std::vector<float> t2s_session_get_ref_audio_emb(t2s_session & session, const t2s_model & model) {
    if (session.ref_T_ref <= 0) return {};
    const size_t d = model.hparams.embedding_dim;
    std::vector<float> x((size_t)(session.ref_T_ref + session.ref_T_prompt) * d);
    if (!t2s_embed_input(session, session.ref_tokens.data(), session.ref_bert.data(), (int)session.ref_T_ref,
                         session.ref_codes.data(), (int)session.ref_T_prompt, x.data()))
        return {};
    return std::vector<float>(x.begin() + (ptrdiff_t)(session.ref_T_ref * d), x.end());
}

// Prefill rows f32 [T_ref + T_in + T_prompt][d_model] (host) for an input text after the reference.
inline bool t2s_embed_with_ref(t2s_session & session, const t2s_model & model, const int32_t * phones,
                               const float * bert, int T_in, std::vector<float> & x_out) {
    T2S_CUDA_ASSERT(session.ref_T_ref > 0, "t2s_session_compute_ref_emb was not called");
    const int T_text = (int)session.ref_T_ref + T_in;
    std::vector<int32_t> ph(session.ref_tokens);
    ph.insert(ph.end(), phones, phones + T_in);
    std::vector<float> bt(session.ref_bert);
    bt.insert(bt.end(), bert, bert + (size_t)T_in * 1024);
    x_out.assign((size_t)(T_text + session.ref_T_prompt) * model.hparams.embedding_dim, 0.0f);
    return t2s_embed_input(session, ph.data(), bt.data(), T_text, session.ref_codes.data(), (int)session.ref_T_prompt,
                           x_out.data());
}

// ---- flex plans (t2s.h:496-582) ----
struct t2s_batch_plan {
    std::vector<int> n_query;   // size n_batch; 0 = slot idle this step
    int total() const {
        int t = 0;
        for (int q : n_query) t += q;
        return t;
    }
};

struct t2s_flex_graph {
    std::vector<float>   x_prefill;         // {N_prefill x d_model}, prefill slots in slot order (caller fills)
    std::vector<int32_t> decode_token_ids;  // {n_decode}, decode slots in slot order (caller fills)
    std::vector<int32_t> sampled;           // {n_active} output, active slots in slot order
    std::vector<int32_t> greedy;            // {n_active} output
    std::vector<int>     prefill_slots, decode_slots, prefill_nq;
    int N = 0, n_active = 0, n_decode = 0, d_model = 0;
    bool built = false, advanced = false;
};

inline t2s_flex_graph t2s_session_build_flex_graph(t2s_session & session, const t2s_model & model,
                                                   const t2s_batch_plan & plan) {
    t2s_flex_graph g;
    if (!session.handle || plan.n_query.size() != session.n_batch) {
        std::fprintf(stderr, "t2s_session_build_flex_graph: plan size %zu != n_batch %u\n", plan.n_query.size(),
                     session.n_batch);
        return g;
    }
    g.d_model = (int)model.hparams.embedding_dim;
    int n_prefill_rows = 0;
    for (uint32_t i = 0; i < session.n_batch; ++i) {
        const int nq = plan.n_query[i];
        if (nq <= 0) continue;
        if (t2sx_session_slot_n_pos(session.handle, (int32_t)i) > 0) {
            g.decode_slots.push_back((int)i);
        } else {
            g.prefill_slots.push_back((int)i);
            g.prefill_nq.push_back(nq);
            n_prefill_rows += nq;
        }
    }
    g.N = plan.total();
    g.n_decode = (int)g.decode_slots.size();
    g.n_active = g.n_decode + (int)g.prefill_slots.size();
    g.x_prefill.assign((size_t)n_prefill_rows * g.d_model, 0.0f);
    g.decode_token_ids.assign(g.n_decode, 0);
    g.sampled.assign(g.n_active, 0);
    g.greedy.assign(g.n_active, 0);
    g.built = true;
    return g;
}

inline void t2s_flex_graph_free(t2s_flex_graph & graph) { graph = t2s_flex_graph(); }

// Validates the plan against the slot states (the reference's asserts, session.cpp:712-859).
inline void t2s_session_flex_advance(t2s_session & session, const t2s_batch_plan & plan, t2s_flex_graph & graph) {
    T2S_CUDA_ASSERT(graph.built, "graph not built");
    T2S_CUDA_ASSERT(graph.N == plan.total(), "plan changed since the graph was built");
    T2S_CUDA_ASSERT(plan.n_query.size() == session.n_batch, "plan size != n_batch");
    for (size_t k = 0; k < graph.decode_slots.size(); ++k) {
        const int i = graph.decode_slots[k];
        T2S_CUDA_ASSERT(plan.n_query[i] == 1, "a decode slot takes exactly one query token");
        T2S_CUDA_ASSERT(t2sx_session_slot_n_pos(session.handle, i) < (int)session.slot_size, "slot is full");
    }
    for (size_t k = 0; k < graph.prefill_slots.size(); ++k) {
        const int i = graph.prefill_slots[k];
        T2S_CUDA_ASSERT(t2sx_session_slot_n_pos(session.handle, i) == 0, "prefill of an active slot");
        T2S_CUDA_ASSERT(plan.n_query[i] <= (int)session.slot_size, "prefill longer than slot_size");
        T2S_CUDA_ASSERT(plan.n_query[i] >= session.ref_T_prompt,
                        "prefill n_query < ref_T_prompt (audio_offset would be negative)");
    }
    // a plan that decodes must decode every active slot: the decode path steps all of them
    // (prefill-only plans leave the active slots alone)
    for (uint32_t i = 0; graph.n_decode > 0 && i < session.n_batch; ++i)
        if (t2sx_session_slot_n_pos(session.handle, (int32_t)i) > 0)
            T2S_CUDA_ASSERT(plan.n_query[i] == 1, "an active slot left idle in a decoding plan (the decode path steps every active slot)");
    graph.advanced = true;
}

// Runs the plan (replaces ggml_backend_graph_compute on the flex graph): one decode step of the
// active slots, then the prefill of the new ones.  sampled / greedy come in slot order.
inline bool t2s_flex_graph_compute(t2s_session & session, t2s_flex_graph & graph) {
    T2S_CUDA_ASSERT(graph.advanced, "t2s_session_flex_advance was not called");
    graph.advanced = false;
    std::vector<std::pair<int, int>> out;   // (slot, token) / greedy
    std::vector<std::pair<int, int>> outg;
    int64_t rows = graph.n_decode;
    for (int v : graph.prefill_nq) rows += v;
    if (rows <= 32768) {   // the whole plan in one pass
        const int nd = graph.n_decode, np = (int)graph.prefill_slots.size();
        std::vector<int32_t> ds(graph.decode_slots.begin(), graph.decode_slots.begin() + nd);
        std::vector<int32_t> dt(graph.decode_token_ids.begin(), graph.decode_token_ids.begin() + nd);
        std::vector<int32_t> ps(graph.prefill_slots.begin(), graph.prefill_slots.end());
        std::vector<int32_t> nq(graph.prefill_nq.begin(), graph.prefill_nq.end()), tp(np, (int32_t)session.ref_T_prompt);
        std::vector<int32_t> tok(nd + np), gr(nd + np);
        if (t2sx_flex_step(session.handle, nd, ds.data(), dt.data(), np, ps.data(), nq.data(), tp.data(),
                           np ? graph.x_prefill.data() : nullptr, tok.data()) != T2SX_OK) {
            std::fprintf(stderr, "t2s_flex_graph_compute: %s\n", t2sx_last_error());
            return false;
        }
        int32_t nr = 0;
        t2sx_read_greedy(session.handle, gr.data(), nd + np, &nr);
        for (int k = 0; k < nd + np; ++k) {
            const int sl = k < nd ? ds[k] : ps[k - nd];
            out.push_back({sl, tok[k]});
            outg.push_back({sl, gr[k]});
        }
    } else if (graph.n_decode > 0) {
        std::vector<int32_t> tok(graph.n_decode), gr(graph.n_decode);
        if (t2sx_decode_step_host(session.handle, graph.decode_token_ids.data(), tok.data()) != T2SX_OK) {
            std::fprintf(stderr, "t2s_flex_graph_compute (decode): %s\n", t2sx_last_error());
            return false;
        }
        int32_t rows = 0;
        t2sx_read_greedy(session.handle, gr.data(), graph.n_decode, &rows);
        for (int k = 0; k < graph.n_decode; ++k) { out.push_back({graph.decode_slots[k], tok[k]}); outg.push_back({graph.decode_slots[k], gr[k]}); }
    }
    if (rows > 32768 && !graph.prefill_slots.empty()) {
        const int n = (int)graph.prefill_slots.size();
        std::vector<int32_t> slots(graph.prefill_slots.begin(), graph.prefill_slots.end());
        std::vector<int32_t> nq(graph.prefill_nq.begin(), graph.prefill_nq.end()), tp(n, (int32_t)session.ref_T_prompt);
        std::vector<int32_t> tok(n), gr(n);
        if (t2sx_prefill(session.handle, n, slots.data(), nq.data(), tp.data(), graph.x_prefill.data(), 0, tok.data()) != T2SX_OK) {
            std::fprintf(stderr, "t2s_flex_graph_compute (prefill): %s\n", t2sx_last_error());
            return false;
        }
        int32_t rows = 0;
        t2sx_read_greedy(session.handle, gr.data(), n, &rows);
        for (int k = 0; k < n; ++k) { out.push_back({slots[k], tok[k]}); outg.push_back({slots[k], gr[k]}); }
    }
    // slot order
    for (size_t a = 0; a < out.size(); ++a)
        for (size_t b = a + 1; b < out.size(); ++b)
            if (out[b].first < out[a].first) { std::swap(out[a], out[b]); std::swap(outg[a], outg[b]); }
    for (size_t k = 0; k < out.size(); ++k) { graph.sampled[k] = out[k].second; graph.greedy[k] = outg[k].second; }
    return true;
}

// ---- persistent decode graph (t2s.h:415,477-488) ----
inline bool t2s_session_build_decode_graph(t2s_session & session, const t2s_model & model) {
    if (!session.handle || !model.handle) {
        std::fprintf(stderr, "t2s_session_build_decode_graph: session or model not initialised\n");
        return false;
    }
    session.decode_ready = true;
    return true;
}

// All n_batch slots must be active, with room for one more position (session.cpp:247-284).
inline void t2s_session_decode_advance(t2s_session & session) {
    T2S_CUDA_ASSERT(session.decode_ready, "decode graph not built");
    for (uint32_t i = 0; i < session.n_batch; ++i) {
        const int n_pos = t2sx_session_slot_n_pos(session.handle, (int32_t)i);
        T2S_CUDA_ASSERT(n_pos > 0, "decode of an idle slot");
        T2S_CUDA_ASSERT(n_pos < (int)session.slot_size, "slot is full");
    }
    session.advanced = true;
}

// One decode step (replaces ggml_backend_graph_compute on the decode graph): token_id -> sampled.
inline bool t2s_session_decode_compute(t2s_session & session) {
    T2S_CUDA_ASSERT(session.advanced, "t2s_session_decode_advance was not called");
    session.advanced = false;
    if (t2sx_decode_step_host(session.handle, session.token_id.data(), session.sampled.data()) != T2SX_OK) {
        std::fprintf(stderr, "t2s_session_decode_compute: %s\n", t2sx_last_error());
        return false;
    }
    int32_t rows = 0;
    t2sx_read_greedy(session.handle, session.greedy.data(), (int32_t)session.n_batch, &rows);
    return true;
}

// Sampler inputs (t2s_session_get_seen_mask / get_exp_noise): one slot's seen mask
// (uint8 [vocab], nonzero = seen); Exp(1) noise for the next passes, rows x vocab (nullptr = greedy).
inline bool t2s_session_set_seen_mask(t2s_session & session, int slot_id, const uint8_t * seen) {
    return t2sx_set_seen(session.handle, slot_id, seen) == T2SX_OK;
}
inline bool t2s_session_set_exp_noise(t2s_session & session, const float * noise, int rows) {
    return t2sx_set_exp_noise(session.handle, noise, rows) == T2SX_OK;
}

}  // namespace gpt_sovits

#endif
