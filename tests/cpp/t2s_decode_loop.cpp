// The reference's decode loop (tests/t2s/test_t2s_infer.cpp:204-421 of GPT-SoVITS.cpp) against
// include/gpt_sovits/t2s.h, with the same calls in the same order: each prompt is prefilled by a
// one-slot flex plan (ref_T_prompt set on the session first), then the persistent decode graph
// runs: ggml_backend_tensor_set(token_id, seen_mask), t2s_session_decode_advance,
// ggml_backend_graph_compute, ggml_backend_tensor_get(sampled, greedy).  Then one mixed plan
// (slot 0 released and prefilled again while the other slots decode) and more decode steps.
//
// usage: t2s_decode_loop MODEL.gguf INPUTS.bin N_STEPS OUT_PREFIX [mode]
//   mode: release_bad | decode_idle | prefill_busy (each must abort), or
//         ref HUBERT.bin (reference embedding: prompt 0 is the reference text, HUBERT.bin
//         int32 T_hub + f32 [T_hub][768]; prompt 1's text follows it; slot 0 prefilled)
// INPUTS.bin: int32 n, then per prompt: int32 T_text, int32 T_prompt, int32 phones[T_text],
// f32 bert[T_text][1024], int32 sem[T_prompt]; the last prompt refills slot 0 in the mixed plan.
// Prints one JSON object; writes OUT_PREFIX.y (flex y of the first prefill, f32) and
// OUT_PREFIX.k0 (slot 0's layer-0 K cache after it, f16 bits).
#include <gpt_sovits/t2s.h>
#include <ggml-cuda.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace gpt_sovits;

struct Prompt {
    int T_text = 0, T_prompt = 0;
    std::vector<int32_t> phones, sem;
    std::vector<float> bert;
};

static bool read_inputs(const char* path, std::vector<Prompt>& out) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    int32_t n = 0;
    bool ok = std::fread(&n, 4, 1, f) == 1;
    for (int i = 0; ok && i < n; ++i) {
        Prompt p;
        ok = std::fread(&p.T_text, 4, 1, f) == 1 && std::fread(&p.T_prompt, 4, 1, f) == 1;
        if (!ok) break;
        p.phones.resize(p.T_text); p.bert.resize((size_t)p.T_text * 1024); p.sem.resize(p.T_prompt);
        ok = std::fread(p.phones.data(), 4, p.T_text, f) == (size_t)p.T_text &&
             std::fread(p.bert.data(), 4, p.bert.size(), f) == p.bert.size() &&
             std::fread(p.sem.data(), 4, p.T_prompt, f) == (size_t)p.T_prompt;
        out.push_back(std::move(p));
    }
    std::fclose(f);
    return ok;
}

static void write_file(const std::string& path, const void* data, size_t bytes) {
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f || std::fwrite(data, 1, bytes, f) != bytes) std::exit(11);
    std::fclose(f);
}

// One flex plan: slot `slot` prefilled with x (rows of the prompt), and, when decode_others, every
// other active slot decoding its current token.  Returns the plan's sampled tokens by slot.
static std::vector<int> run_plan(t2s_session& s, const t2s_model& m, ggml_backend_t backend, int slot,
                                 const std::vector<float>& x, int T_prompt, const std::vector<int>& cur,
                                 bool decode_others, std::vector<float>* y_out) {
    s.ref_T_prompt = T_prompt;   // the reference tests set the public field before the plan
    t2s_batch_plan plan;
    plan.n_query.assign(s.n_batch, 0);
    plan.n_query[slot] = (int)(x.size() / m.hparams.hidden_dim);
    for (uint32_t i = 0; decode_others && i < s.n_batch; ++i)
        if ((int)i != slot && t2s_session_slot_n_pos(s, (int)i) > 0) plan.n_query[i] = 1;
    t2s_flex_graph g = t2s_session_build_flex_graph(s, m, plan);
    if (!g.ctx || g.N != plan.total()) std::exit(4);
    ggml_backend_tensor_set(g.x_prefill, x.data(), 0, x.size() * sizeof(float));
    if (g.n_decode > 0) {
        std::vector<int32_t> ids;
        for (uint32_t i = 0; i < s.n_batch; ++i)
            if (plan.n_query[i] == 1) ids.push_back(cur[i]);
        ggml_backend_tensor_set(g.decode_token_ids, ids.data(), 0, ids.size() * sizeof(int32_t));
    }
    std::vector<float> zeros((size_t)m.hparams.vocab_size * g.n_active, 0.0f);
    ggml_backend_tensor_set(g.seen_mask, zeros.data(), 0, zeros.size() * sizeof(float));
    t2s_session_flex_advance(s, plan, g);
    if (ggml_backend_graph_compute(backend, g.gf) != GGML_STATUS_SUCCESS) std::exit(5);
    std::vector<int32_t> sampled(g.n_active), greedy(g.n_active);
    ggml_backend_tensor_get(g.sampled, sampled.data(), 0, sampled.size() * sizeof(int32_t));
    ggml_backend_tensor_get(g.greedy, greedy.data(), 0, greedy.size() * sizeof(int32_t));
    if (sampled != greedy) std::exit(12);   // no noise set: the greedy pick
    if (y_out) {
        y_out->resize((size_t)m.hparams.hidden_dim * g.N);
        ggml_backend_tensor_get(g.y, y_out->data(), 0, y_out->size() * sizeof(float));
    }
    std::vector<int> tok(s.n_batch, -1);
    for (uint32_t i = 0, k = 0; i < s.n_batch; ++i)
        if (plan.n_query[i] > 0) tok[i] = sampled[k++];
    t2s_flex_graph_free(g);
    return tok;
}

int main(int argc, char** argv) {
    if (argc < 5) { std::fprintf(stderr, "usage: %s MODEL INPUTS N_STEPS OUT_PREFIX [mode]\n", argv[0]); return 2; }
    const char* mode = argc > 5 ? argv[5] : "";
    const std::string out_prefix = argv[4];
    std::vector<Prompt> prompts;
    if (!read_inputs(argv[2], prompts) || prompts.size() < 2) { std::fprintf(stderr, "bad inputs\n"); return 2; }
    const int n_steps = std::atoi(argv[3]);
    const int n = (int)prompts.size() - 1;   // sessions; the last prompt refills slot 0

    ggml_backend_t backend = ggml_backend_cuda_init(0);
    if (!backend) return 1;
    t2s_model model;
    if (!t2s_model_load(argv[1], model, backend)) return 1;
    const int d = (int)model.hparams.hidden_dim, V = (int)model.hparams.vocab_size;
    int slot_size = 0;
    for (auto& p : prompts) slot_size = std::max(slot_size, p.T_text + p.T_prompt);
    slot_size += 2 * n_steps + 2;
    if (!std::strcmp(mode, "ref")) slot_size *= 3;   // reference text + input text + prompt codes
    t2s_sampler_config cfg;
    cfg.repetition_penalty = 1.0f;
    cfg.eos_mask = true;
    t2s_session session;
    if (t2s_session_init(session, model.hparams, backend, (uint32_t)n, (uint32_t)slot_size, cfg)) return 13;   // F32 KV: refused
    if (!t2s_session_init(session, model.hparams, backend, (uint32_t)n, (uint32_t)slot_size, cfg, GGML_TYPE_F16)) return 1;

    if (!std::strcmp(mode, "ref")) {
        if (argc < 7) return 2;
        FILE* f = std::fopen(argv[6], "rb");
        int32_t T_hub = 0;
        if (!f || std::fread(&T_hub, 4, 1, f) != 1) return 2;
        std::vector<float> hub((size_t)T_hub * 768);
        const bool ok = std::fread(hub.data(), 4, hub.size(), f) == hub.size();
        std::fclose(f);
        if (!ok) return 2;
        const Prompt& ref = prompts[0];
        if (!t2s_session_compute_ref_emb(session, model, ref.phones.data(), ref.T_text, ref.bert.data(), hub.data(), T_hub))
            return 8;
        if (t2s_session_get_ref_T_ref(session) != ref.T_text) return 9;
        const int64_t T_prompt = t2s_session_get_ref_T_prompt(session);
        std::vector<float> x;
        if (!t2s_session_build_prefill_input(session, model, prompts[1].phones.data(), prompts[1].T_text,
                                             prompts[1].bert.data(), x))
            return 3;
        std::vector<int> cur(session.n_batch, 0);
        const std::vector<int> tok = run_plan(session, model, backend, 0, x, (int)T_prompt, cur, false, nullptr);
        ggml_tensor* te = t2s_session_get_ref_text_emb(session);
        ggml_tensor* ae = t2s_session_get_ref_audio_emb(session);
        if (!te || !ae || te->ne[0] != d || te->ne[1] != ref.T_text || ae->ne[1] != T_prompt) return 10;
        std::vector<float> tv((size_t)ggml_nelements(te)), av((size_t)ggml_nelements(ae));
        ggml_backend_tensor_get(te, tv.data(), 0, ggml_nbytes(te));
        ggml_backend_tensor_get(ae, av.data(), 0, ggml_nbytes(ae));
        write_file(out_prefix + ".text", tv.data(), tv.size() * 4);
        write_file(out_prefix + ".audio", av.data(), av.size() * 4);
        std::printf("{\"T_prompt\": %lld, \"tokens\": [%d]}\n", (long long)T_prompt, tok[0]);
        t2s_session_free(session);
        t2s_model_free(model);
        ggml_backend_free(backend);
        return 0;
    }
    if (!std::strcmp(mode, "release_bad")) t2s_session_slot_release(session, n);   // aborts
    if (!std::strcmp(mode, "decode_idle")) {                                        // aborts
        t2s_session_build_decode_graph(session, model);
        t2s_session_decode_advance(session);
    }

    // ---- phase 1: prefill each prompt through a one-slot flex plan ----
    std::vector<int> cur(n, 0), first(n);
    for (int i = 0; i < n; ++i) {
        const int slot = t2s_session_find_free_slot(session);
        if (slot != i) { std::fprintf(stderr, "unexpected free slot %d\n", slot); return 6; }
        const Prompt& p = prompts[i];
        std::vector<float> x((size_t)(p.T_text + p.T_prompt) * d);
        if (!t2s_session_embed_input(session, model, p.phones.data(), p.bert.data(), p.T_text, p.sem.data(), p.T_prompt,
                                     x.data()))
            return 3;
        std::vector<float> y;
        first[i] = run_plan(session, model, backend, slot, x, p.T_prompt, cur, false, i == 0 ? &y : nullptr)[slot];
        cur[i] = first[i];
        if (i == 0) {
            write_file(out_prefix + ".y", y.data(), y.size() * 4);
            const t2s_layer_caches lc = t2s_session_get_layer_caches(session, 0);
            std::vector<uint16_t> k((size_t)t2s_session_slot_n_pos(session, 0) * d);
            ggml_backend_tensor_get(lc.k, k.data(), 0, k.size() * 2);
            write_file(out_prefix + ".k0", k.data(), k.size() * 2);
        }
    }
    if (!std::strcmp(mode, "prefill_busy")) {   // aborts: a prefill plan on an active slot
        std::vector<float> x((size_t)(prompts[0].T_text + prompts[0].T_prompt) * d, 0.0f);
        run_plan(session, model, backend, 0, x, prompts[0].T_prompt, cur, false, nullptr);
    }

    // ---- phase 2: the persistent decode graph ----
    if (!t2s_session_build_decode_graph(session, model)) return 1;
    ggml_tensor* tok_t = t2s_session_get_token_id(session);
    ggml_tensor* seen_t = t2s_session_get_seen_mask(session);
    ggml_tensor* pos_t = t2s_session_get_position(session);
    if (!tok_t || !seen_t || !pos_t || !t2s_session_get_exp_noise(session)) return 7;
    std::vector<float> seen((size_t)V * n, 0.0f);
    std::vector<std::vector<int>> steps;
    auto run_steps = [&](int k) {
        for (int st = 0; st < k; ++st) {
            std::vector<int32_t> ids(cur.begin(), cur.end());
            ggml_backend_tensor_set(tok_t, ids.data(), 0, ids.size() * sizeof(int32_t));
            ggml_backend_tensor_set(seen_t, seen.data(), 0, seen.size() * sizeof(float));
            t2s_session_decode_advance(session);
            if (ggml_backend_graph_compute(backend, t2s_session_get_decode_graph(session)) != GGML_STATUS_SUCCESS) std::exit(7);
            std::vector<int32_t> sampled(n), greedy(n);
            ggml_backend_tensor_get(t2s_session_get_sampled(session), sampled.data(), 0, n * sizeof(int32_t));
            ggml_backend_tensor_get(t2s_session_get_greedy(session), greedy.data(), 0, n * sizeof(int32_t));
            for (int i = 0; i < n; ++i) {
                if (sampled[i] < 0 || sampled[i] >= V) std::exit(14);
                seen[(size_t)i * V + sampled[i]] = 1.0f;
            }
            steps.emplace_back(sampled.begin(), sampled.end());
            cur.assign(sampled.begin(), sampled.end());
        }
    };
    run_steps(n_steps);
    // ---- phase 3: slot 0 released and refilled with the last prompt while the others decode ----
    t2s_session_slot_release(session, 0);
    const Prompt& p = prompts[n];
    std::vector<float> x((size_t)(p.T_text + p.T_prompt) * d);
    if (!t2s_session_embed_input(session, model, p.phones.data(), p.bert.data(), p.T_text, p.sem.data(), p.T_prompt, x.data()))
        return 3;
    const std::vector<int> mixed_tok = run_plan(session, model, backend, 0, x, p.T_prompt, cur, true, nullptr);
    std::vector<int> mixed(mixed_tok.begin(), mixed_tok.end());
    cur = mixed;
    run_steps(n_steps);
    // the decode mask's column 0 reveals exactly slot 0's written positions
    const int64_t max_ctx = t2s_session_get_n_kv(session);
    std::vector<uint16_t> col((size_t)max_ctx);
    ggml_backend_tensor_get(t2s_session_get_mask(session), col.data(), 0, col.size() * 2);
    const int visible = (int)std::count(col.begin(), col.end(), (uint16_t)0);

    std::printf("{\"first\": [");
    for (int i = 0; i < n; ++i) std::printf("%s%d", i ? ", " : "", first[i]);
    std::printf("], \"mixed\": [");
    for (int i = 0; i < n; ++i) std::printf("%s%d", i ? ", " : "", mixed[i]);
    std::printf("], \"mask_visible_slot0\": %d, \"n_pos_slot0\": %d, \"steps\": [", visible, t2s_session_slot_n_pos(session, 0));
    for (size_t k = 0; k < steps.size(); ++k) {
        std::printf("%s[", k ? ", " : "");
        for (size_t i = 0; i < steps[k].size(); ++i) std::printf("%s%d", i ? ", " : "", steps[k][i]);
        std::printf("]");
    }
    std::printf("]}\n");
    t2s_session_free(session);
    t2s_session_free(session);   // idempotent, as in the reference
    t2s_model_free(model);
    t2s_model_free(model);
    ggml_backend_free(backend);
    return 0;
}
