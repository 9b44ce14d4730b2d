// The reference's decode loop (tests/t2s/test_t2s_infer.cpp:204-421 of GPT-SoVITS.cpp) written
// against the C++ session layer (include/gpt_sovits/t2s_cuda.h): prefill each prompt through a
// prefill-only flex plan, then step the persistent decode graph, then one mixed plan (a slot
// released and prefilled again while the other slots decode), then more decode steps.
//
// usage: t2s_decode_loop MODEL.gguf INPUTS.bin N_STEPS [release_bad|decode_idle|plan_idle]
//        t2s_decode_loop MODEL.gguf INPUTS.bin N_STEPS ref HUBERT.bin [EMB_PREFIX]
// ref: prompt 0 is the reference text, HUBERT.bin (int32 T_hub, f32 [T_hub][768]) its audio
// features; t2s_session_compute_ref_emb extracts the prompt codes, prompt 1's text is embedded
// after the reference, slot 0 is prefilled and decoded; prints the codes and the tokens.
// INPUTS.bin: int32 n, then per prompt: int32 T_text, int32 T_prompt, int32 phones[T_text],
// f32 bert[T_text][1024], int32 sem[T_prompt]; the last prompt refills slot 0 in the mixed plan.
// Prints one JSON object with the sampled tokens.
#include <gpt_sovits/t2s_cuda.h>

#include <algorithm>
#include <cstdio>
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

// prefill one prompt into `slot` with a prefill-only plan; returns the first sampled token
static int prefill_one(t2s_session& s, const t2s_model& m, int slot, const Prompt& p, int decode_others) {
    const int nq = p.T_text + p.T_prompt;
    std::vector<float> x((size_t)nq * m.hparams.embedding_dim);
    if (!t2s_embed_input(s, p.phones.data(), p.bert.data(), p.T_text, p.sem.data(), p.T_prompt, x.data())) std::exit(3);
    s.ref_T_prompt = p.T_prompt;
    t2s_batch_plan plan;
    plan.n_query.assign(s.n_batch, 0);
    plan.n_query[slot] = nq;
    for (uint32_t i = 0; decode_others && i < s.n_batch; ++i)
        if ((int)i != slot && t2s_session_slot_n_pos(s, (int)i) > 0) plan.n_query[i] = 1;
    t2s_flex_graph g = t2s_session_build_flex_graph(s, m, plan);
    if (!g.built) std::exit(4);
    std::memcpy(g.x_prefill.data(), x.data(), x.size() * sizeof(float));
    for (int k = 0; k < g.n_decode; ++k) g.decode_token_ids[k] = s.token_id[g.decode_slots[k]];
    t2s_session_flex_advance(s, plan, g);
    if (!t2s_flex_graph_compute(s, g)) std::exit(5);
    int tok = -1, k = 0;
    for (uint32_t i = 0; i < s.n_batch; ++i) {
        if (plan.n_query[i] == 0) continue;
        if ((int)i == slot) tok = g.sampled[k];
        else s.token_id[i] = g.sampled[k];   // decoded slots continue from their new token
        ++k;
    }
    t2s_flex_graph_free(g);
    return tok;
}

int main(int argc, char** argv) {
    if (argc < 4) { std::fprintf(stderr, "usage: %s MODEL INPUTS N_STEPS [mode]\n", argv[0]); return 2; }
    const char* mode = argc > 4 ? argv[4] : "";
    std::vector<Prompt> prompts;
    if (!read_inputs(argv[2], prompts) || prompts.size() < 2) { std::fprintf(stderr, "bad inputs\n"); return 2; }
    const int n_steps = std::atoi(argv[3]);
    const int n = (int)prompts.size() - 1;   // sessions; the last prompt refills slot 0

    t2s_model model;
    if (!t2s_model_load(argv[1], model, 0)) return 1;
    int slot_size = 0;
    for (auto& p : prompts) slot_size = std::max(slot_size, p.T_text + p.T_prompt);
    slot_size += 2 * n_steps + 2;
    if (!std::strcmp(mode, "ref")) slot_size *= 3;   // reference text + input text + prompt codes
    t2s_session session;
    t2s_sampler_config cfg;
    cfg.repetition_penalty = 1.0f;
    if (!t2s_session_init(session, model, (uint32_t)n, (uint32_t)slot_size, cfg, /*eos_mask=*/true)) return 1;

    if (!std::strcmp(mode, "ref")) {
        if (argc < 6) return 2;
        FILE* f = std::fopen(argv[5], "rb");
        int32_t T_hub = 0;
        if (!f || std::fread(&T_hub, 4, 1, f) != 1) return 2;
        std::vector<float> hub((size_t)T_hub * 768);
        const bool ok = std::fread(hub.data(), 4, hub.size(), f) == hub.size();
        std::fclose(f);
        if (!ok) return 2;
        const Prompt& ref = prompts[0];
        if (!t2s_session_compute_ref_emb(session, model, ref.phones.data(), ref.T_text, ref.bert.data(), hub.data(),
                                         T_hub))
            return 8;
        if (t2s_session_get_ref_T_ref(session) != ref.T_text) return 9;
        std::vector<float> x;
        if (!t2s_embed_with_ref(session, model, prompts[1].phones.data(), prompts[1].bert.data(), prompts[1].T_text, x))
            return 3;
        t2s_batch_plan plan;
        plan.n_query.assign(session.n_batch, 0);
        plan.n_query[0] = (int)(x.size() / model.hparams.embedding_dim);
        t2s_flex_graph g = t2s_session_build_flex_graph(session, model, plan);
        if (!g.built) return 4;
        std::memcpy(g.x_prefill.data(), x.data(), x.size() * sizeof(float));
        t2s_session_flex_advance(session, plan, g);
        if (!t2s_flex_graph_compute(session, g)) return 5;
        const int tok = g.sampled[0];
        t2s_flex_graph_free(g);
        if (t2s_session_get_n_kv(session) != (int)(session.n_batch * session.slot_size)) return 10;
        if (argc > 6) {   // the cached reference embeddings, raw f32
            const std::vector<float> te = t2s_session_get_ref_text_emb(session, model);
            const std::vector<float> ae = t2s_session_get_ref_audio_emb(session, model);
            const std::string base = argv[6];
            FILE* ft = std::fopen((base + ".text").c_str(), "wb");
            FILE* fa = std::fopen((base + ".audio").c_str(), "wb");
            if (!ft || !fa) return 11;
            std::fwrite(te.data(), 4, te.size(), ft);
            std::fwrite(ae.data(), 4, ae.size(), fa);
            std::fclose(ft);
            std::fclose(fa);
        }
        std::printf("{\"codes\": [");
        for (size_t i = 0; i < session.ref_codes.size(); ++i) std::printf("%s%d", i ? ", " : "", session.ref_codes[i]);
        std::printf("], \"T_prompt\": %lld, \"tokens\": [", (long long)t2s_session_get_ref_T_prompt(session));
        std::printf("%d]}\n", tok);
        t2s_session_free(session);
        t2s_model_free(model);
        return 0;
    }
    if (!std::strcmp(mode, "release_bad")) t2s_session_slot_release(session, n);   // aborts
    if (!std::strcmp(mode, "decode_idle")) {                                        // aborts
        t2s_session_build_decode_graph(session, model);
        t2s_session_decode_advance(session);
    }

    std::vector<int> first(n);
    for (int i = 0; i < n; ++i) {
        const int slot = t2s_session_find_free_slot(session);
        if (slot != i) { std::fprintf(stderr, "unexpected free slot %d\n", slot); return 6; }
        first[i] = prefill_one(session, model, slot, prompts[i], 0);
        session.token_id[slot] = first[i];
    }
    if (!std::strcmp(mode, "plan_idle")) {   // aborts: a decoding plan that leaves an active slot idle
        t2s_batch_plan plan;
        plan.n_query.assign(session.n_batch, 0);
        plan.n_query[0] = 1;
        t2s_flex_graph g = t2s_session_build_flex_graph(session, model, plan);
        t2s_session_flex_advance(session, plan, g);
    }

    if (!t2s_session_build_decode_graph(session, model)) return 1;
    std::vector<std::vector<int>> steps;
    auto run_steps = [&](int k) {
        for (int s = 0; s < k; ++s) {
            t2s_session_decode_advance(session);
            if (!t2s_session_decode_compute(session)) std::exit(7);
            steps.emplace_back(session.sampled.begin(), session.sampled.end());
            session.token_id = session.sampled;
        }
    };
    run_steps(n_steps);
    // mixed plan: slot 0 released and refilled with the last prompt while the others decode
    t2s_session_slot_release(session, 0);
    const int refill = prefill_one(session, model, 0, prompts[n], 1);
    std::vector<int> mixed(session.token_id.begin(), session.token_id.end());
    mixed[0] = refill;
    session.token_id[0] = refill;
    run_steps(n_steps);

    std::printf("{\"first\": [");
    for (int i = 0; i < n; ++i) std::printf("%s%d", i ? ", " : "", first[i]);
    std::printf("], \"mixed\": [");
    for (int i = 0; i < n; ++i) std::printf("%s%d", i ? ", " : "", mixed[i]);
    std::printf("], \"steps\": [");
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
    return 0;
}
