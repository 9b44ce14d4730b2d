// T2S decode-path oracle -- TEST INFRASTRUCTURE ONLY.
//
// A CPU restatement of the arithmetic of GPT-SoVITS.cpp's T2S path (src/t2s/block.cpp,
// src/t2s/session.cpp) as executed by the ggml CPU backend, written from the operator
// definitions.  It is the checker for the CUDA library: only tests/, the smoke entry and
// the cpu_baseline leg of bench.py load it.  Nothing in the product links or calls it.
//
// Parity status (see the header of t2s_oracle.cpp for the per-op detail):
//   * pinned   : GGUF tensor layout and the Q8_0/Q4_0/Q4_K/F16 dequantisation (bit-exact against
//                gguf-py's dequantize), the session bookkeeping (kv positions, masks, n_pos,
//                audio_offset) against the reference's own known-answer unit tests.
//   * unpinned : the float summation order of ggml's SIMD kernels (ggml is an empty submodule in
//                the reference snapshot and cannot be built or run); the oracle fixes one order,
//                documented per op, and the CUDA kernels reproduce that order bit for bit.
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// ggml type ids used by the GGUF files (ggml.h enum ggml_type).
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q5_0 = 6, ORC_Q8_0 = 8, ORC_Q4_K = 12 };

// ---- primitives -------------------------------------------------------------------------
float    orc_expf(float x);
uint16_t orc_f32_to_f16(float x);
float    orc_f16_to_f32(uint16_t h);
int64_t  orc_row_bytes(int type, int64_t n);
// Activation quantisation into ggml block bytes (Q8_0: 34 B / 32; Q8_K: 292 B / 256).
void     orc_quantize_q8_0(const float* x, int64_t n, uint8_t* out);
void     orc_quantize_q8_K(const float* x, int64_t n, uint8_t* out);
// Weight quantisation helpers (used to build synthetic GGUFs and tests).
void     orc_dequantize(int type, const void* data, int64_t n, float* out);
// y[m][n] = W[n] . x[m]  (no bias), W in ggml block layout, canonical order.
int      orc_matmul(int wtype, const void* w, int64_t N, int64_t K,
                    const float* x, int64_t M, float* y);
// One head of attention.  q f32[32]; k,v f16 [L][32]; out f32[32].
void     orc_attn_decode(const float* q, const uint16_t* k, const uint16_t* v, int L, float* out);
// Batched rows over per-sequence caches k, v: f16 bits [n_seqs][max_len][16][32].  Row r: q f16
// bits [n][512], every head attends to positions [0, lens[r]) of sequence seqs[r]; out f32 [n][512].
// 32 position lanes merged by the xor butterfly, as for every attention row.
void     orc_attn_rows(int n, const int* seqs, const int* lens, const uint16_t* q16, const uint16_t* k,
                       const uint16_t* v, int max_len, float* out);
void     orc_layernorm(const float* x, const float* g, const float* b, int n, float eps, float* y);
void     orc_pe_row(int pos, int d_model, float* out);

// ---- model / session --------------------------------------------------------------------
void*    orc_model_load(const char* path);
void     orc_model_free(void* model);
// hp[0..8] = embedding_dim, hidden_dim, n_head, linear_units, n_layer, vocab_size,
//            phoneme_vocab_size, eos, inter_channels; types[0] = qkv_w type.
int      orc_model_info(void* model, uint32_t* hp, int32_t* types);

void*    orc_session_new(void* model, int n_slots, int capacity);
void     orc_session_free(void* sess);
void     orc_set_threads(int n);
// Prefill embedding (block.cpp:424-511): text rows from phone ids + BERT features, audio rows
// from semantic ids, PE from position 0 for each part.  x_out f32 [T_text + T_prompt][d].
int      orc_embed_prefill(void* model, const int32_t* phones, const float* bert, int T_text,
                           const int32_t* sem, int T_prompt, float* x_out);
// Prefill one slot with nq rows of x (f32 [nq][d]); T_prompt drives the mask and audio_offset.
// Writes the slot's greedy token and (optionally) its logits f32 [vocab].
int      orc_prefill(void* sess, int slot, const float* x, int nq, int T_prompt, int eos_mask,
                     int32_t* token_out, float* logits_out, float* y_out);
// One decode step over n slots (tokens_in[i] embedded at slot[i]).  seen: f32 [n][vocab] or null.
int      orc_decode_step(void* sess, int n, const int32_t* slots, const int32_t* tokens_in,
                         const float* seen, float rep_penalty, int eos_mask,
                         int32_t* tokens_out, float* logits_out);
// Decode step with the full sampler (noise f32 [n][vocab] by sorted position, or null).
int      orc_decode_step2(void* sess, int n, const int32_t* slots, const int32_t* tokens_in,
                          const float* seen, const float* noise, int top_k, float top_p,
                          float temperature, float rp, int eos_mask, int32_t* sampled_out,
                          int32_t* greedy_out, float* logits_out);
int      orc_slot_n_pos(void* sess, int slot);
// Evaluation order of the session (before its first prefill; -1 otherwise).  ggml_order is a
// mask of operators that follow ggml's CPU operator definitions instead of the canonical order
// the CUDA kernels reproduce: 1 the matmuls (generic vec_dot folds), 2 LayerNorm (sequential
// double sums), 4 flash attention (per-query sequential fold, f16 V accumulator, libm expf); 7 =
// all.  kv_f32 = 1 keeps an F32 KV cache (the reference's default kv_cache_type: f32 query and V
// accumulator; implies 7).
int      orc_session_set_mode(void* sess, int ggml_order, int kv_f32);
// The matmul with ggml's generic vec_dot folds (see orc_session_set_mode).
int      orc_matmul_ggml(int wtype, const void* w, int64_t N, int64_t K,
                         const float* x, int64_t M, float* y);
// Extract-latent codes of HuBERT frames f32 [T][768]: writes (T - 2) / 2 + 1 codes, returns that
// count (-1 on a missing tensor or T < 2).
int      orc_extract_latent(void* model, const float* hubert, int T, int32_t* codes_out);
// t2s_session_slot_release (session.cpp:224-240): the slot becomes idle (n_pos = 0).
int      orc_slot_release(void* sess, int slot);
// Sampler chain (block.cpp:52-348) on n rows of logits f32 [n][vocab]; seen f32 [n][vocab] or
// null; noise f32 [n][vocab] Exp(1) samples indexed by sorted position, or null (greedy).
int      orc_sample(void* model, int n, const float* logits, const float* seen, const float* noise,
                    int top_k, float top_p, float temperature, float rp, int eos_mask,
                    int32_t* sampled, int32_t* greedy);
// Read back the slot's cached K or V (f16) of one layer: [n_pos][d].
int      orc_read_kv(void* sess, int slot, int layer, int which, uint16_t* out);

#ifdef __cplusplus
}
#endif
