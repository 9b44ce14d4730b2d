// The reference-compatible T2S interface (include/gpt_sovits/t2s.h) and the ggml type shim
// (include/ggml*.h) over the C ABI of libt2sx (include/t2sx.h).
//
// Session semantics follow src/t2s/session.cpp of the reference: the host mirror of slot state
// (n_pos, audio_offset, kv_pos, positions, the decode mask) is updated by decode_advance /
// flex_advance / slot_release exactly as there, and ggml_backend_graph_compute then runs the
// step on the device through t2sx_decode_step_host / t2sx_flex_step, whose own host-side checks
// agree with the mirror.  Tensors are views: inputs and outputs live in host buffers owned by
// the session (or flex graph), KV caches and masks are materialised from device state when read.
#include "../../include/gpt_sovits/t2s.h"
#include "../../include/ggml-cuda.h"
#include "../../include/t2sx.h"

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <string>
#include <vector>

// ============================================================================================
// ggml type shim
// ============================================================================================
struct ggml_backend {
    int device;
    char name[48];
};

// kind 1: a session's decode step (owner = t2s_session_impl); kind 2: a flex plan (owner = FlexImpl)
struct ggml_cgraph {
    int kind;
    void* owner;
};

namespace {

enum TensorKind { K_HOST = 0, K_KCACHE = 1, K_VCACHE = 2, K_DEC_MASK = 3, K_FLEX_MASK = 4, K_WEIGHT = 5 };
// roles of host tensors whose writes the owner tracks
enum TensorRole { R_NONE = 0, R_SEEN = 1, R_NOISE = 2, R_FLEX_SEEN = 3, R_FLEX_NOISE = 4 };

struct TypeInfo { int64_t blck; size_t size; const char* name; };
TypeInfo type_info(enum ggml_type t) {
    switch (t) {
        case GGML_TYPE_F32: return {1, 4, "f32"};
        case GGML_TYPE_F16: return {1, 2, "f16"};
        case GGML_TYPE_Q4_0: return {32, 18, "q4_0"};
        case GGML_TYPE_Q4_1: return {32, 20, "q4_1"};
        case GGML_TYPE_Q5_0: return {32, 22, "q5_0"};
        case GGML_TYPE_Q5_1: return {32, 24, "q5_1"};
        case GGML_TYPE_Q8_0: return {32, 34, "q8_0"};
        case GGML_TYPE_Q8_1: return {32, 36, "q8_1"};
        case GGML_TYPE_Q4_K: return {256, 144, "q4_K"};
        case GGML_TYPE_I32: return {1, 4, "i32"};
    }
    return {1, 0, "unknown"};
}

// Tensors and host storage of one owner (model, session, flex graph); addresses stay stable.
struct TensorStore {
    std::deque<ggml_tensor> tensors;
    std::deque<std::vector<uint8_t>> bufs;
    ggml_tensor* make(enum ggml_type type, const int64_t* ne, int nd, const char* name, int kind, int index, void* owner,
                      bool host) {
        tensors.emplace_back();
        ggml_tensor* t = &tensors.back();
        std::memset(t, 0, sizeof(*t));
        t->type = type;
        for (int i = 0; i < GGML_MAX_DIMS; ++i) t->ne[i] = i < nd ? ne[i] : 1;
        const TypeInfo ti = type_info(type);
        t->nb[0] = ti.size;
        t->nb[1] = ti.size * (size_t)(t->ne[0] / ti.blck);
        for (int i = 2; i < GGML_MAX_DIMS; ++i) t->nb[i] = t->nb[i - 1] * (size_t)t->ne[i - 1];
        std::snprintf(t->name, sizeof(t->name), "%s", name);
        t->t2s_kind = kind;
        t->t2s_index = index;
        t->t2s_owner = owner;
        if (host) {
            bufs.emplace_back(ggml_nbytes(t), 0);
            t->data = bufs.back().data();
        }
        return t;
    }
    ggml_tensor* host2(enum ggml_type type, int64_t ne0, int64_t ne1, const char* name, int role, void* owner) {
        const int64_t ne[2] = {ne0, ne1};
        return make(type, ne, 2, name, K_HOST, role, owner, true);
    }
};

[[noreturn]] void die(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::fprintf(stderr, "t2s: ");
    std::vfprintf(stderr, fmt, ap);
    std::fprintf(stderr, "\n");
    va_end(ap);
    std::abort();
}

const ggml_fp16_t kF16Zero = 0x0000, kF16NegInf = 0xFC00;

}  // namespace

extern "C" {

int64_t ggml_nelements(const struct ggml_tensor* t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

size_t ggml_nbytes(const struct ggml_tensor* t) {
    const TypeInfo ti = type_info(t->type);
    return (size_t)(t->ne[0] / ti.blck) * ti.size * (size_t)(t->ne[1] * t->ne[2] * t->ne[3]);
}

size_t ggml_type_size(enum ggml_type type) { return type_info(type).size; }
int64_t ggml_blck_size(enum ggml_type type) { return type_info(type).blck; }
const char* ggml_type_name(enum ggml_type type) { return type_info(type).name; }

float ggml_fp16_to_fp32(ggml_fp16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1f, man = h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        float v = (float)man * 5.9604644775390625e-08f;   // subnormal: man * 2^-24
        std::memcpy(&u, &v, 4);
        u |= sign;
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

ggml_fp16_t ggml_fp32_to_fp16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t au = u & 0x7fffffffu;
    if (au >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (au > 0x7f800000u ? 0x200u : 0u));
    if (au >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    const int e = (int)(au >> 23) - 127;
    if (e >= -14) {   // normal: round half to even on the 13 dropped bits
        uint32_t val = ((uint32_t)(e + 15) << 10) | ((au & 0x7fffffu) >> 13);
        const uint32_t rem = au & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (val & 1u))) val += 1;
        return (uint16_t)(sign | val);
    }
    if (e < -25) return sign;
    const uint32_t man = (au & 0x7fffffu) | 0x800000u;
    const int shift = -e - 1;
    uint32_t q = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q += 1;
    return (uint16_t)(sign | q);
}

void ggml_abort(const char* file, int line, const char* fmt, ...) {
    std::fprintf(stderr, "%s:%d: ", file, line);
    va_list ap;
    va_start(ap, fmt);
    std::vfprintf(stderr, fmt, ap);
    va_end(ap);
    std::fprintf(stderr, "\n");
    std::abort();
}

ggml_backend_t ggml_backend_cuda_init(int device) {
    int32_t n = 0;
    if (t2sx_device_count(&n) != T2SX_OK || device < 0 || device >= n) return nullptr;
    ggml_backend* b = new ggml_backend();
    b->device = device;
    std::snprintf(b->name, sizeof(b->name), "CUDA%d", device);
    return b;
}

int ggml_backend_cuda_get_device_count(void) {
    int32_t n = 0;
    return t2sx_device_count(&n) == T2SX_OK ? n : 0;
}

const char* ggml_backend_name(ggml_backend_t backend) { return backend ? backend->name : "(null)"; }

void ggml_backend_free(ggml_backend_t backend) { delete backend; }

}  // extern "C"

// ============================================================================================
// session state
// ============================================================================================
namespace gpt_sovits {

struct ModelImpl {
    TensorStore store;
};

struct t2s_session_impl {
    int device = 0;
    uint32_t n_batch = 0, slot_size = 0, d = 512, vocab = 0, n_layer = 0;
    t2s_sampler_config cfg;
    t2sx_session* h = nullptr;        // created with the model at the first use that passes one
    const t2sx_model* mh = nullptr;
    std::vector<int> n_pos, audio_off;   // the reference's slot state (mirrored into t2s_session::slots)
    bool keep_mask_host = false;
    TensorStore store;
    ggml_tensor *kv_pos = nullptr, *mask = nullptr, *token_id = nullptr, *position = nullptr, *pe_table = nullptr,
                *seen = nullptr, *noise = nullptr, *sampled = nullptr, *greedy = nullptr;
    std::vector<ggml_tensor*> kc, vc;
    uint64_t seen_ver = 0, seen_done = 0, noise_ver = 0;
    bool noise_loaded = false;           // exp noise currently set on the device session
    bool dec_built = false;
    int pending_advance = 0;
    ggml_cgraph dec_graph{1, nullptr};
    // reference embedding
    std::vector<int32_t> ref_tokens, ref_codes;
    std::vector<float> ref_bert;
    ggml_tensor *ref_text = nullptr, *ref_audio = nullptr;
};

struct FlexImpl {
    t2s_session_impl* s = nullptr;
    TensorStore store;
    ggml_cgraph graph{2, nullptr};
    std::vector<int> nq;                        // the plan
    std::vector<int32_t> dec_slots, pre_slots, pre_nq, pre_tp;   // in slot order
    std::vector<int> act_slots;                 // active slots in slot order
    std::vector<int> q_slot, q_len;             // per query row (slot order): slot, visible prefix
    int N = 0, n_active = 0, n_decode = 0, n_prefill_rows = 0;
    bool advanced = false;
    uint64_t seen_ver = 0, noise_ver = 0;
    ggml_tensor *x_prefill = nullptr, *dec_tok = nullptr, *dec_pos = nullptr, *kv_pos = nullptr, *mask = nullptr,
                *y = nullptr, *seen = nullptr, *noise = nullptr, *sampled = nullptr, *greedy = nullptr;
};

static void sync_slots(t2s_session& session) {
    t2s_session_impl* S = session.impl;
    session.slots.resize(S->n_batch);
    for (uint32_t i = 0; i < S->n_batch; ++i) {
        session.slots[i].n_pos = S->n_pos[i];
        session.slots[i].audio_offset = S->audio_off[i];
    }
}

// The device session, created with the model at the first call that passes one.
static bool ensure_device(t2s_session& session, const t2s_model& model, const char* who) {
    t2s_session_impl* S = session.impl;
    if (!S || !model.handle) {
        std::fprintf(stderr, "%s: session or model not initialised\n", who);
        return false;
    }
    if (S->h) {
        if (S->mh != model.handle) {
            std::fprintf(stderr, "%s: the session is bound to another model\n", who);
            return false;
        }
        return true;
    }
    t2sx_sampler_config c{S->cfg.top_k, S->cfg.top_p, S->cfg.temperature, S->cfg.repetition_penalty, S->cfg.eos_mask ? 1 : 0};
    if (t2sx_session_create(model.handle, S->n_batch, S->slot_size, &c, &S->h) != T2SX_OK) {
        std::fprintf(stderr, "%s: %s\n", who, t2sx_last_error());
        S->h = nullptr;
        return false;
    }
    S->mh = model.handle;
    return true;
}

// ---- model ----
bool t2s_model_load(const std::string& fname, t2s_model& model, ggml_backend_t backend) {
    GGML_ASSERT(backend != nullptr);
    t2s_model_free(model);
    t2sx_model* h = nullptr;
    if (t2sx_model_load(fname.c_str(), backend->device, &h) != T2SX_OK) {
        std::fprintf(stderr, "t2s_model_load: %s\n", t2sx_last_error());
        return false;
    }
    uint32_t hp[9];
    int32_t wt[4];
    t2sx_model_hparams(h, hp, wt);
    model.hparams = t2s_hparams{hp[0], hp[1], hp[2], hp[3], hp[4], hp[5], hp[6], hp[7], hp[8]};
    ModelImpl* mi = new ModelImpl();
    auto w = [&](const std::string& name) -> ggml_tensor* {
        int32_t type = 0, nd = 0;
        int64_t ne[4] = {1, 1, 1, 1};
        if (t2sx_model_tensor_info(h, name.c_str(), &type, &nd, ne) != T2SX_OK) return nullptr;
        return mi->store.make((enum ggml_type)type, ne, nd, name.c_str(), K_WEIGHT, 0, mi, false);
    };
    t2s_model_weights& W = model.weights;
    W.extract_latent = {w("extract_latent.ssl_proj_w"), w("extract_latent.ssl_proj_b"), w("extract_latent.codebook")};
    W.embed = {w("encoder.text_embedding"), w("encoder.bert_proj_w"), w("encoder.bert_proj_b"),
               w("encoder.text_pos_alpha"), w("encoder.audio_embedding"), w("encoder.audio_pos_alpha")};
    W.attention.clear();
    for (uint32_t i = 0; i < model.hparams.n_layer; ++i) {
        const std::string p = "attention." + std::to_string(i) + ".";
        W.attention.push_back({w(p + "qkv_w"), w(p + "qkv_b"), w(p + "out_proj_w"), w(p + "out_proj_b"), w(p + "ln1_w"),
                               w(p + "ln1_b"), w(p + "ffn_up_w"), w(p + "ffn_up_b"), w(p + "ffn_down_w"),
                               w(p + "ffn_down_b"), w(p + "ln2_w"), w(p + "ln2_b")});
    }
    W.lm_head_w = w("sampler.lm_head_w");
    model.backend = backend;
    model.ctx_w = reinterpret_cast<ggml_context*>(mi);
    model.buf_w = nullptr;
    model.handle = h;
    return true;
}

void t2s_model_free(t2s_model& model) {
    if (model.handle) t2sx_model_free(model.handle);   // released after its last session
    delete reinterpret_cast<ModelImpl*>(model.ctx_w);
    model.handle = nullptr;
    model.ctx_w = nullptr;
    model.buf_w = nullptr;
    model.backend = nullptr;
    model.weights = t2s_model_weights{};
}

// ---- session ----
bool t2s_session_init(t2s_session& session, const t2s_hparams& hparams, ggml_backend_t backend, uint32_t n_batch,
                      uint32_t slot_size, const t2s_sampler_config& sampler_cfg, enum ggml_type kv_cache_type) {
    GGML_ASSERT(backend != nullptr);
    if (n_batch == 0 || slot_size == 0) {
        std::fprintf(stderr, "t2s_session_init: n_batch and slot_size must be > 0\n");
        return false;
    }
    if (kv_cache_type != GGML_TYPE_F16) {
        std::fprintf(stderr, "t2s_session_init: kv_cache_type %s is not supported: this implementation keeps an f16 KV "
                             "cache (pass GGML_TYPE_F16)\n", type_info(kv_cache_type).name);
        return false;
    }
    t2s_session_free(session);
    t2s_session_impl* S = new t2s_session_impl();
    S->device = backend->device;
    S->n_batch = n_batch;
    S->slot_size = slot_size;
    S->d = hparams.hidden_dim;
    S->vocab = hparams.vocab_size;
    S->n_layer = hparams.n_layer;
    S->cfg = sampler_cfg;
    S->n_pos.assign(n_batch, 0);
    S->audio_off.assign(n_batch, 0);
    S->dec_graph.owner = S;
    const int64_t max_ctx = (int64_t)n_batch * slot_size;
    for (uint32_t l = 0; l < S->n_layer; ++l) {
        const int64_t ne[2] = {S->d, max_ctx};
        S->kc.push_back(S->store.make(GGML_TYPE_F16, ne, 2, "k_cache", K_KCACHE, (int)l, S, false));
        S->vc.push_back(S->store.make(GGML_TYPE_F16, ne, 2, "v_cache", K_VCACHE, (int)l, S, false));
    }
    S->kv_pos = S->store.host2(GGML_TYPE_I32, n_batch, 1, "kv_pos", R_NONE, S);
    {
        const int64_t ne[2] = {max_ctx, n_batch};
        S->mask = S->store.make(GGML_TYPE_F16, ne, 2, "mask", K_DEC_MASK, 0, S, false);
    }
    S->token_id = S->store.host2(GGML_TYPE_I32, n_batch, 1, "token_id", R_NONE, S);
    S->position = S->store.host2(GGML_TYPE_I32, n_batch, 1, "position", R_NONE, S);
    S->pe_table = S->store.host2(GGML_TYPE_F32, S->d, slot_size, "pe_table", R_NONE, S);
    {   // the reference's PE table (session.cpp:33-53), same expression
        float* pe = (float*)S->pe_table->data;
        const int64_t half = S->d / 2;
        std::vector<float> freq(half);
        for (int64_t j = 0; j < half; ++j) freq[j] = std::exp(-std::log((float)10000) * (float)j / (float)half);
        for (int64_t p = 0; p < (int64_t)slot_size; ++p)
            for (int64_t j = 0; j < half; ++j) {
                const float arg = (float)p * freq[j];
                pe[p * S->d + 2 * j] = std::sin(arg);
                pe[p * S->d + 2 * j + 1] = std::cos(arg);
            }
    }
    S->seen = S->store.host2(GGML_TYPE_F32, S->vocab, n_batch, "seen_mask", R_SEEN, S);
    S->noise = S->store.host2(GGML_TYPE_F32, S->vocab, n_batch, "exp_noise", R_NOISE, S);
    S->sampled = S->store.host2(GGML_TYPE_I32, n_batch, 1, "sampled", R_NONE, S);
    S->greedy = S->store.host2(GGML_TYPE_I32, n_batch, 1, "greedy", R_NONE, S);
    S->keep_mask_host = (double)max_ctx * n_batch <= (double)(1 << 24);

    session.n_batch = n_batch;
    session.slot_size = slot_size;
    session.kv_cache_type = kv_cache_type;
    session.backend = backend;
    session.sampler_cfg = sampler_cfg;
    session.impl = S;
    session.ctx_kv = reinterpret_cast<ggml_context*>(S);
    session.k_caches = S->kc;
    session.v_caches = S->vc;
    session.kv_pos = S->kv_pos;
    session.mask = S->mask;
    session.token_id = S->token_id;
    session.position = S->position;
    session.pe_table = S->pe_table;
    session.seen_mask = S->seen;
    session.exp_noise = S->noise;
    session.sampled = S->sampled;
    session.greedy = S->greedy;
    session.mask_host.assign(S->keep_mask_host ? (size_t)max_ctx * n_batch : 0, kF16NegInf);
    session.ref_T_ref = session.ref_T_prompt = 0;
    sync_slots(session);
    return true;
}

void t2s_session_free(t2s_session& session) {
    t2s_session_impl* S = session.impl;
    if (S) {
        if (S->h) t2sx_session_free(S->h);
        delete S;
    }
    session = t2s_session();
}

int t2s_session_find_free_slot(const t2s_session& session) {
    for (size_t i = 0; i < session.slots.size(); ++i)
        if (session.slots[i].n_pos == 0) return (int)i;
    return -1;
}

void t2s_session_slot_release(t2s_session& session, int slot_id) {
    GGML_ASSERT(session.impl != nullptr);
    GGML_ASSERT(slot_id >= 0 && (size_t)slot_id < session.slots.size());
    t2s_session_impl* S = session.impl;
    if (S->keep_mask_host) {
        const int64_t max_ctx = (int64_t)S->n_batch * S->slot_size;
        for (uint32_t k = 0; k < S->slot_size; ++k)
            session.mask_host[slot_id * max_ctx + (int64_t)slot_id * S->slot_size + k] = kF16NegInf;
    }
    if (S->h && S->n_pos[slot_id] > 0 && t2sx_session_slot_release(S->h, slot_id) != T2SX_OK)
        die("t2s_session_slot_release: %s", t2sx_last_error());
    S->n_pos[slot_id] = 0;
    S->audio_off[slot_id] = 0;
    sync_slots(session);
}

int t2s_session_slot_n_pos(const t2s_session& session, int slot_id) {
    GGML_ASSERT(slot_id >= 0 && (size_t)slot_id < session.slots.size());
    return session.slots[slot_id].n_pos;
}

void t2s_session_decode_advance(t2s_session& session) {
    GGML_ASSERT(session.impl != nullptr);
    t2s_session_impl* S = session.impl;
    // the persistent decode step processes every slot (session.cpp:247-284)
    for (uint32_t i = 0; i < S->n_batch; ++i) GGML_ASSERT(S->n_pos[i] > 0);
    GGML_ASSERT(S->pending_advance == 0 && "t2s_session_decode_advance called twice without a decode step");
    const int64_t max_ctx = (int64_t)S->n_batch * S->slot_size;
    int32_t* kvp = (int32_t*)S->kv_pos->data;
    int32_t* pos = (int32_t*)S->position->data;
    for (uint32_t i = 0; i < S->n_batch; ++i) {
        GGML_ASSERT(S->n_pos[i] < (int)S->slot_size);
        const int row = (int)(i * S->slot_size) + S->n_pos[i];
        if (S->keep_mask_host) session.mask_host[i * max_ctx + row] = kF16Zero;
        kvp[i] = row;
        GGML_ASSERT(S->audio_off[i] >= 0 && S->audio_off[i] < (int)S->slot_size && "decode on slot with invalid audio_offset");
        const int pe_pos = S->n_pos[i] - S->audio_off[i];
        GGML_ASSERT(pe_pos >= 0 && pe_pos < (int)S->slot_size && "decode PE position out of pe_table bounds");
        pos[i] = pe_pos;
        S->n_pos[i] += 1;
    }
    S->pending_advance = 1;
    sync_slots(session);
}

t2s_layer_caches t2s_session_get_layer_caches(const t2s_session& session, int layer) {
    GGML_ASSERT(layer >= 0 && (size_t)layer < session.k_caches.size());
    return {session.k_caches[layer], session.v_caches[layer]};
}
ggml_tensor* t2s_session_get_kv_pos(const t2s_session& session) { return session.kv_pos; }
ggml_tensor* t2s_session_get_mask(const t2s_session& session) { return session.mask; }
int t2s_session_get_n_kv(const t2s_session& session) { return (int)(session.n_batch * session.slot_size); }

// ---- reference embedding ----
bool t2s_session_compute_ref_emb(t2s_session& session, const t2s_model& model, const int32_t* ref_token, int64_t T_ref,
                                 const float* ref_bert, const float* hubert_data, int64_t T_hub) {
    if (!ensure_device(session, model, "t2s_session_compute_ref_emb")) return false;
    if (!ref_token || !ref_bert || !hubert_data || T_ref <= 0 || T_hub < 2) {
        std::fprintf(stderr, "t2s_session_compute_ref_emb: bad inputs (T_ref=%lld, T_hub=%lld)\n", (long long)T_ref,
                     (long long)T_hub);
        return false;
    }
    t2s_session_impl* S = session.impl;
    std::vector<int32_t> codes((size_t)((T_hub - 2) / 2 + 1));
    if (t2sx_extract_latent(S->h, hubert_data, (int32_t)T_hub, codes.data()) != T2SX_OK) {
        std::fprintf(stderr, "t2s_session_compute_ref_emb: %s\n", t2sx_last_error());
        return false;
    }
    const int64_t T_prompt = (int64_t)codes.size();
    std::vector<float> x((size_t)(T_ref + T_prompt) * S->d);
    if (t2sx_embed_prefill(S->h, ref_token, ref_bert, (int32_t)T_ref, codes.data(), (int32_t)T_prompt, x.data(), 0) != T2SX_OK) {
        std::fprintf(stderr, "t2s_session_compute_ref_emb: %s\n", t2sx_last_error());
        return false;
    }
    S->ref_tokens.assign(ref_token, ref_token + T_ref);
    S->ref_bert.assign(ref_bert, ref_bert + T_ref * 1024);
    S->ref_codes = codes;
    S->ref_text = S->store.host2(GGML_TYPE_F32, S->d, T_ref, "ref_text_emb", R_NONE, S);
    S->ref_audio = S->store.host2(GGML_TYPE_F32, S->d, T_prompt, "ref_audio_emb", R_NONE, S);
    std::memcpy(S->ref_text->data, x.data(), (size_t)T_ref * S->d * 4);
    std::memcpy(S->ref_audio->data, x.data() + (size_t)T_ref * S->d, (size_t)T_prompt * S->d * 4);
    session.ref_text_emb = S->ref_text;
    session.ref_audio_emb = S->ref_audio;
    session.ref_T_ref = T_ref;
    session.ref_T_prompt = T_prompt;
    return true;
}
ggml_tensor* t2s_session_get_ref_text_emb(const t2s_session& session) { return session.ref_text_emb; }
ggml_tensor* t2s_session_get_ref_audio_emb(const t2s_session& session) { return session.ref_audio_emb; }
int64_t t2s_session_get_ref_T_ref(const t2s_session& session) { return session.ref_T_ref; }
int64_t t2s_session_get_ref_T_prompt(const t2s_session& session) { return session.ref_T_prompt; }

bool t2s_session_embed_input(t2s_session& session, const t2s_model& model, const int32_t* phones, const float* bert,
                             int64_t T_text, const int32_t* sem, int64_t T_prompt, float* x_out) {
    if (!ensure_device(session, model, "t2s_session_embed_input")) return false;
    if (t2sx_embed_prefill(session.impl->h, phones, bert, (int32_t)T_text, sem, (int32_t)T_prompt, x_out, 0) != T2SX_OK) {
        std::fprintf(stderr, "t2s_session_embed_input: %s\n", t2sx_last_error());
        return false;
    }
    return true;
}

bool t2s_session_build_prefill_input(t2s_session& session, const t2s_model& model, const int32_t* input_token,
                                     int64_t T_in, const float* input_bert, std::vector<float>& x_out) {
    t2s_session_impl* S = session.impl;
    if (!S || S->ref_tokens.empty()) {
        std::fprintf(stderr, "t2s_session_build_prefill_input: t2s_session_compute_ref_emb was not called\n");
        return false;
    }
    std::vector<int32_t> ph(S->ref_tokens);
    ph.insert(ph.end(), input_token, input_token + T_in);
    std::vector<float> bt(S->ref_bert);
    bt.insert(bt.end(), input_bert, input_bert + T_in * 1024);
    const int64_t T_text = (int64_t)ph.size(), T_prompt = (int64_t)S->ref_codes.size();
    x_out.assign((size_t)(T_text + T_prompt) * S->d, 0.0f);
    return t2s_session_embed_input(session, model, ph.data(), bt.data(), T_text, S->ref_codes.data(), T_prompt,
                                   x_out.data());
}

// ---- decode step ----
bool t2s_session_build_decode_graph(t2s_session& session, const t2s_model& model) {
    if (!ensure_device(session, model, "t2s_session_build_decode_graph")) return false;
    session.impl->dec_built = true;
    session.gf_dec = &session.impl->dec_graph;
    session.ctx_graph = reinterpret_cast<ggml_context*>(session.impl);
    return true;
}
ggml_tensor* t2s_session_get_token_id(const t2s_session& session) { return session.token_id; }
ggml_tensor* t2s_session_get_position(const t2s_session& session) { return session.position; }
ggml_cgraph* t2s_session_get_decode_graph(const t2s_session& session) { return session.gf_dec; }
ggml_tensor* t2s_session_get_sampled(const t2s_session& session) { return session.sampled; }
ggml_tensor* t2s_session_get_greedy(const t2s_session& session) { return session.greedy; }
ggml_tensor* t2s_session_get_seen_mask(const t2s_session& session) { return session.seen_mask; }
ggml_tensor* t2s_session_get_exp_noise(const t2s_session& session) { return session.exp_noise; }

// seen rows (f32, > 0 = seen) of the given slots onto the device session, when the penalty uses them
static bool upload_seen(t2s_session_impl* S, const float* rows, const int32_t* slots, int n) {
    if (S->cfg.repetition_penalty == 1.0f) return true;
    std::vector<uint8_t> b(S->vocab);
    for (int r = 0; r < n; ++r) {
        for (uint32_t v = 0; v < S->vocab; ++v) b[v] = rows[(size_t)r * S->vocab + v] > 0.0f ? 1 : 0;
        if (t2sx_set_seen(S->h, slots[r], b.data()) != T2SX_OK) return false;
    }
    return true;
}

static enum ggml_status compute_decode(t2s_session_impl* S) {
    if (!S->dec_built) die("ggml_backend_graph_compute: the decode graph was not built");
    if (S->pending_advance != 1) die("ggml_backend_graph_compute: t2s_session_decode_advance was not called before the decode step");
    S->pending_advance = 0;
    std::vector<int32_t> all(S->n_batch);
    for (uint32_t i = 0; i < S->n_batch; ++i) all[i] = (int32_t)i;
    if (S->seen_ver != S->seen_done) {
        if (!upload_seen(S, (const float*)S->seen->data, all.data(), (int)S->n_batch)) goto fail;
        S->seen_done = S->seen_ver;
    }
    if (S->noise_ver > 0) {   // the stochastic chain once the caller supplies noise
        if (t2sx_set_exp_noise(S->h, (const float*)S->noise->data, (int32_t)S->n_batch) != T2SX_OK) goto fail;
        S->noise_loaded = true;
    } else if (S->noise_loaded) {
        if (t2sx_set_exp_noise(S->h, nullptr, 0) != T2SX_OK) goto fail;
        S->noise_loaded = false;
    }
    if (t2sx_decode_step_host(S->h, (const int32_t*)S->token_id->data, (int32_t*)S->sampled->data) != T2SX_OK) goto fail;
    {
        int32_t rows = 0;
        if (t2sx_read_greedy(S->h, (int32_t*)S->greedy->data, (int32_t)S->n_batch, &rows) != T2SX_OK) goto fail;
    }
    return GGML_STATUS_SUCCESS;
fail:
    std::fprintf(stderr, "ggml_backend_graph_compute (decode step): %s\n", t2sx_last_error());
    return GGML_STATUS_FAILED;
}

// ---- flex plans ----
t2s_flex_graph t2s_session_build_flex_graph(t2s_session& session, const t2s_model& model, const t2s_batch_plan& plan) {
    t2s_flex_graph g;
    const int N = plan.total();
    if (N <= 0) {
        std::fprintf(stderr, "t2s_session_build_flex_graph: plan has no tokens (total=%d)\n", N);
        return g;
    }
    if (plan.n_query.size() != session.n_batch) {
        std::fprintf(stderr, "t2s_session_build_flex_graph: plan size (%zu) != n_batch (%u)\n", plan.n_query.size(),
                     session.n_batch);
        return g;
    }
    if (!ensure_device(session, model, "t2s_session_build_flex_graph")) return g;
    t2s_session_impl* S = session.impl;
    FlexImpl* F = new FlexImpl();
    F->s = S;
    F->graph.owner = F;
    F->nq = plan.n_query;
    F->N = N;
    for (uint32_t i = 0; i < S->n_batch; ++i) {
        const int q = plan.n_query[i];
        if (q <= 0) continue;
        F->act_slots.push_back((int)i);
        if (q == 1) F->dec_slots.push_back((int32_t)i);
        else { F->pre_slots.push_back((int32_t)i); F->pre_nq.push_back(q); F->n_prefill_rows += q; }
    }
    F->n_active = (int)F->act_slots.size();
    F->n_decode = (int)F->dec_slots.size();
    const int64_t n_kv = (int64_t)S->n_batch * S->slot_size;
    if (F->n_prefill_rows > 0) F->x_prefill = F->store.host2(GGML_TYPE_F32, S->d, F->n_prefill_rows, "x_prefill", R_NONE, F);
    if (F->n_decode > 0) {
        F->dec_tok = F->store.host2(GGML_TYPE_I32, F->n_decode, 1, "decode_token_ids", R_NONE, F);
        F->dec_pos = F->store.host2(GGML_TYPE_I32, F->n_decode, 1, "decode_positions", R_NONE, F);
    }
    F->kv_pos = F->store.host2(GGML_TYPE_I32, N, 1, "kv_pos", R_NONE, F);
    {
        const int64_t ne[2] = {n_kv, N};
        F->mask = F->store.make(GGML_TYPE_F16, ne, 2, "mask", K_FLEX_MASK, 0, F, false);
    }
    F->y = F->store.host2(GGML_TYPE_F32, S->d, N, "y", R_NONE, F);
    F->seen = F->store.host2(GGML_TYPE_F32, S->vocab, F->n_active, "seen_mask", R_FLEX_SEEN, F);
    F->noise = F->store.host2(GGML_TYPE_F32, S->vocab, F->n_active, "exp_noise", R_FLEX_NOISE, F);
    F->sampled = F->store.host2(GGML_TYPE_I32, F->n_active, 1, "sampled", R_NONE, F);
    F->greedy = F->store.host2(GGML_TYPE_I32, F->n_active, 1, "greedy", R_NONE, F);
    g.x_prefill = F->x_prefill;
    g.decode_token_ids = F->dec_tok;
    g.decode_positions = F->dec_pos;
    g.kv_pos = F->kv_pos;
    g.mask = F->mask;
    g.y = F->y;
    g.seen_mask = F->seen;
    g.exp_noise = F->noise;
    g.sampled = F->sampled;
    g.greedy = F->greedy;
    g.ctx = reinterpret_cast<ggml_context*>(F);
    g.gf = &F->graph;
    g.backend = session.backend;
    g.N = N;
    g.n_active = F->n_active;
    g.n_decode = F->n_decode;
    return g;
}

void t2s_flex_graph_free(t2s_flex_graph& graph) {
    delete reinterpret_cast<FlexImpl*>(graph.ctx);
    graph = t2s_flex_graph();
}

// The reference's flex_advance (session.cpp:712-859): validation, kv_pos, the attention mask,
// decode PE positions, audio_offset of prefill slots, the persistent decode mask, n_pos.
void t2s_session_flex_advance(t2s_session& session, const t2s_batch_plan& plan, t2s_flex_graph& graph) {
    GGML_ASSERT(graph.ctx != nullptr);
    GGML_ASSERT(graph.N == plan.total());
    GGML_ASSERT(plan.n_query.size() == session.n_batch);
    t2s_session_impl* S = session.impl;
    FlexImpl* F = reinterpret_cast<FlexImpl*>(graph.ctx);
    GGML_ASSERT(F->s == S && F->nq == plan.n_query);
    GGML_ASSERT(!F->advanced && "t2s_session_flex_advance called twice on one graph");
    for (uint32_t i = 0; i < S->n_batch; ++i) {
        const int q = plan.n_query[i];
        if (q <= 0) continue;
        if (q == 1) GGML_ASSERT(S->n_pos[i] > 0);
        else GGML_ASSERT(S->n_pos[i] == 0);
    }
    int32_t* kvp = (int32_t*)F->kv_pos->data;
    F->q_slot.clear();
    F->q_len.clear();
    int off = 0;
    for (uint32_t i = 0; i < S->n_batch; ++i) {
        const int q = plan.n_query[i];
        if (q <= 0) continue;
        GGML_ASSERT(S->n_pos[i] + q <= (int)S->slot_size);
        for (int j = 0; j < q; ++j) kvp[off + j] = (int32_t)(i * S->slot_size) + S->n_pos[i] + j;
        off += q;
        if (q > 1) {
            const int T_text = q - (int)session.ref_T_prompt;
            for (int j = 0; j < q; ++j) {
                F->q_slot.push_back((int)i);
                F->q_len.push_back(std::min((j < T_text) ? T_text : j + 1, (int)S->slot_size));
            }
        } else {
            F->q_slot.push_back((int)i);
            F->q_len.push_back(std::min(S->n_pos[i] + 1, (int)S->slot_size));
        }
    }
    int di = 0;
    F->pre_tp.clear();
    for (uint32_t i = 0; i < S->n_batch; ++i) {
        const int q = plan.n_query[i];
        if (q == 1) {
            GGML_ASSERT(S->audio_off[i] >= 0 && S->audio_off[i] < (int)S->slot_size && "decode on slot with invalid audio_offset");
            const int pe_pos = S->n_pos[i] - S->audio_off[i];
            GGML_ASSERT(pe_pos >= 0 && pe_pos < (int)S->slot_size && "decode PE position out of pe_table bounds");
            ((int32_t*)F->dec_pos->data)[di++] = pe_pos;
        } else if (q > 1) {
            const int offset = q - (int)session.ref_T_prompt;
            GGML_ASSERT(offset >= 0 && "prefill n_query < ref_T_prompt (audio_offset would be negative)");
            S->audio_off[i] = offset;
            F->pre_tp.push_back((int32_t)session.ref_T_prompt);
        }
    }
    const int64_t max_ctx = (int64_t)S->n_batch * S->slot_size;
    for (uint32_t i = 0; i < S->n_batch; ++i) {
        const int q = plan.n_query[i];
        if (q <= 0) continue;
        if (S->keep_mask_host)
            for (int k = 0; k < q; ++k) session.mask_host[i * max_ctx + (int64_t)i * S->slot_size + S->n_pos[i] + k] = kF16Zero;
        S->n_pos[i] += q;
    }
    F->advanced = true;
    sync_slots(session);
}

static enum ggml_status compute_flex(FlexImpl* F) {
    t2s_session_impl* S = F->s;
    if (!F->advanced) die("ggml_backend_graph_compute: t2s_session_flex_advance was not called for this plan");
    F->advanced = false;
    const int nd = F->n_decode, np = (int)F->pre_slots.size(), na = F->n_active;
    // active rows in slot order -> the pass's row order (decode slots, then prefill slots)
    std::vector<int> slot_rank(S->n_batch, -1);
    for (int k = 0; k < na; ++k) slot_rank[F->act_slots[k]] = k;
    std::vector<int> pass_of_act(na);   // active index (slot order) -> pass row
    for (int k = 0; k < nd; ++k) pass_of_act[slot_rank[F->dec_slots[k]]] = k;
    for (int k = 0; k < np; ++k) pass_of_act[slot_rank[F->pre_slots[k]]] = nd + k;
    if (F->seen_ver && nd) {
        std::vector<float> rows((size_t)nd * S->vocab);
        for (int k = 0; k < nd; ++k)
            std::memcpy(&rows[(size_t)k * S->vocab], (const float*)F->seen->data + (size_t)slot_rank[F->dec_slots[k]] * S->vocab,
                        (size_t)S->vocab * 4);
        if (!upload_seen(S, rows.data(), F->dec_slots.data(), nd)) goto fail;
    }
    if (F->noise_ver) {
        std::vector<float> rows((size_t)na * S->vocab);
        for (int k = 0; k < na; ++k)
            std::memcpy(&rows[(size_t)pass_of_act[k] * S->vocab], (const float*)F->noise->data + (size_t)k * S->vocab,
                        (size_t)S->vocab * 4);
        if (t2sx_set_exp_noise(S->h, rows.data(), na) != T2SX_OK) goto fail;
        S->noise_loaded = true;
    } else if (S->noise_loaded) {
        if (t2sx_set_exp_noise(S->h, nullptr, 0) != T2SX_OK) goto fail;
        S->noise_loaded = false;
    }
    {
        std::vector<int32_t> tok(na), gr(na), tok_pass(na), gr_pass(na);
        const int64_t rows_total = (int64_t)nd + F->n_prefill_rows;
        std::vector<float> hid;
        if (rows_total <= 32768) {   // the whole plan in one pass
            if (t2sx_flex_step(S->h, nd, F->dec_slots.data(), nd ? (const int32_t*)F->dec_tok->data : nullptr, np,
                               F->pre_slots.data(), F->pre_nq.data(), F->pre_tp.data(),
                               np ? (const float*)F->x_prefill->data : nullptr, tok_pass.data()) != T2SX_OK)
                goto fail;
            int32_t r = 0;
            if (t2sx_read_greedy(S->h, gr_pass.data(), na, &r) != T2SX_OK) goto fail;
            hid.resize((size_t)rows_total * S->d);
            if (t2sx_read_hidden(S->h, hid.data(), (int32_t)rows_total, &r) != T2SX_OK) goto fail;
        } else {   // decode rows first, then the prefill in chunks (y keeps the decode rows only)
            int32_t r = 0;
            if (nd) {
                if (t2sx_flex_step(S->h, nd, F->dec_slots.data(), (const int32_t*)F->dec_tok->data, 0, nullptr, nullptr,
                                   nullptr, nullptr, tok_pass.data()) != T2SX_OK)
                    goto fail;
                if (t2sx_read_greedy(S->h, gr_pass.data(), nd, &r) != T2SX_OK) goto fail;
                hid.resize((size_t)nd * S->d);
                if (t2sx_read_hidden(S->h, hid.data(), nd, &r) != T2SX_OK) goto fail;
            }
            if (t2sx_prefill(S->h, np, F->pre_slots.data(), F->pre_nq.data(), F->pre_tp.data(),
                             (const float*)F->x_prefill->data, 0, tok_pass.data() + nd) != T2SX_OK)
                goto fail;
            if (t2sx_read_greedy(S->h, gr_pass.data() + nd, np, &r) != T2SX_OK) goto fail;
        }
        for (int k = 0; k < na; ++k) {
            ((int32_t*)F->sampled->data)[k] = tok_pass[pass_of_act[k]];
            ((int32_t*)F->greedy->data)[k] = gr_pass[pass_of_act[k]];
        }
        // y in slot order: each active slot's rows, from the decode rows or its prefill rows
        std::vector<int64_t> pre_row0(np);
        for (int k = 0, r = nd; k < np; ++k) { pre_row0[k] = r; r += F->pre_nq[k]; }
        float* y = (float*)F->y->data;
        int64_t out = 0;
        for (int k = 0; k < na; ++k) {
            const int sl = F->act_slots[k];
            const int q = F->nq[sl];
            const int pr = pass_of_act[k];
            const int64_t src = pr < nd ? pr : pre_row0[pr - nd];
            for (int j = 0; j < q; ++j, ++out) {
                if ((size_t)(src + j + 1) * S->d <= hid.size())
                    std::memcpy(y + out * S->d, hid.data() + (size_t)(src + j) * S->d, (size_t)S->d * 4);
                else
                    std::memset(y + out * S->d, 0, (size_t)S->d * 4);
            }
        }
    }
    return GGML_STATUS_SUCCESS;
fail:
    std::fprintf(stderr, "ggml_backend_graph_compute (flex plan): %s\n", t2sx_last_error());
    return GGML_STATUS_FAILED;
}

}  // namespace gpt_sovits

using gpt_sovits::FlexImpl;
using gpt_sovits::t2s_session_impl;

// ============================================================================================
// tensor access and graph execution
// ============================================================================================
extern "C" {

void ggml_backend_tensor_set(struct ggml_tensor* t, const void* data, size_t offset, size_t size) {
    GGML_ASSERT(t != nullptr);
    if (t->t2s_kind != K_HOST) die("ggml_backend_tensor_set: '%s' is a read-only view of device state", t->name);
    if (offset + size > ggml_nbytes(t) || (size && !data))
        die("ggml_backend_tensor_set: [%zu, %zu) outside '%s' (%zu bytes)", offset, offset + size, t->name, ggml_nbytes(t));
    std::memcpy((uint8_t*)t->data + offset, data, size);
    switch (t->t2s_index) {
        case R_SEEN: ((t2s_session_impl*)t->t2s_owner)->seen_ver++; break;
        case R_NOISE: ((t2s_session_impl*)t->t2s_owner)->noise_ver++; break;
        case R_FLEX_SEEN: ((FlexImpl*)t->t2s_owner)->seen_ver++; break;
        case R_FLEX_NOISE: ((FlexImpl*)t->t2s_owner)->noise_ver++; break;
        default: break;
    }
}

void ggml_backend_tensor_get(const struct ggml_tensor* t, void* data, size_t offset, size_t size) {
    GGML_ASSERT(t != nullptr);
    if (offset + size > ggml_nbytes(t) || (size && !data))
        die("ggml_backend_tensor_get: [%zu, %zu) outside '%s' (%zu bytes)", offset, offset + size, t->name, ggml_nbytes(t));
    uint8_t* dst = (uint8_t*)data;
    switch (t->t2s_kind) {
        case K_HOST:
            std::memcpy(dst, (const uint8_t*)t->data + offset, size);
            return;
        case K_KCACHE:
        case K_VCACHE: {
            // {d_model, n_batch * slot_size} f16: slot i's positions are columns [i*S, i*S + n_pos)
            t2s_session_impl* S = (t2s_session_impl*)t->t2s_owner;
            std::memset(dst, 0, size);
            if (!S->h) return;
            const size_t col_bytes = (size_t)S->d * 2, slot_bytes = col_bytes * S->slot_size;
            std::vector<uint16_t> rows;
            for (uint32_t sl = (uint32_t)(offset / slot_bytes); sl < S->n_batch && (size_t)sl * slot_bytes < offset + size; ++sl) {
                const int n = t2sx_session_slot_n_pos(S->h, (int32_t)sl);
                if (n <= 0) continue;
                rows.assign((size_t)n * S->d, 0);
                if (t2sx_read_kv(S->h, (int32_t)sl, t->t2s_index, t->t2s_kind == K_VCACHE ? 1 : 0, rows.data()) != T2SX_OK)
                    die("ggml_backend_tensor_get: %s", t2sx_last_error());
                const size_t b0 = (size_t)sl * slot_bytes, b1 = b0 + (size_t)n * col_bytes;
                const size_t lo = std::max(b0, offset), hi = std::min(b1, offset + size);
                if (lo < hi) std::memcpy(dst + (lo - offset), (const uint8_t*)rows.data() + (lo - b0), hi - lo);
            }
            return;
        }
        case K_DEC_MASK: {
            // mask(row, col) = 0 where row is a written position of slot col, else -inf
            t2s_session_impl* S = (t2s_session_impl*)t->t2s_owner;
            const int64_t max_ctx = (int64_t)S->n_batch * S->slot_size;
            for (size_t b = offset; b < offset + size; b += 2) {
                const int64_t e = (int64_t)(b / 2), col = e / max_ctx, row = e % max_ctx;
                const int64_t r0 = col * S->slot_size;
                const ggml_fp16_t v = (row >= r0 && row < r0 + S->n_pos[col]) ? kF16Zero : kF16NegInf;
                std::memcpy(dst + (b - offset), &v, 2);
            }
            return;
        }
        case K_FLEX_MASK: {
            FlexImpl* F = (FlexImpl*)t->t2s_owner;
            const int64_t n_kv = t->ne[0];
            for (size_t b = offset; b < offset + size; b += 2) {
                const int64_t e = (int64_t)(b / 2), q = e / n_kv, row = e % n_kv;
                ggml_fp16_t v = kF16NegInf;
                if ((size_t)q < F->q_slot.size()) {
                    const int64_t r0 = (int64_t)F->q_slot[q] * F->s->slot_size;
                    if (row >= r0 && row < r0 + F->q_len[q]) v = kF16Zero;
                }
                std::memcpy(dst + (b - offset), &v, 2);
            }
            return;
        }
        default:
            die("ggml_backend_tensor_get: '%s' is a weight held repacked on the device", t->name);
    }
}

enum ggml_status ggml_backend_graph_compute(ggml_backend_t backend, struct ggml_cgraph* graph) {
    GGML_ASSERT(backend != nullptr && graph != nullptr && graph->owner != nullptr);
    if (graph->kind == 1) return gpt_sovits::compute_decode((t2s_session_impl*)graph->owner);
    if (graph->kind == 2) return gpt_sovits::compute_flex((FlexImpl*)graph->owner);
    die("ggml_backend_graph_compute: unknown graph");
}

}  // extern "C"
