/*
 * t2sx -- C ABI of the B200 T2S decode path (libt2sx.so).
 *
 * Drop-in for the model/session layer of GPT-SoVITS.cpp's T2S path (src/t2s) without a ggml
 * backend: it reads the GGUF files written by python/convert_t2s_to_gguf.py unchanged and runs
 * the prefill and the autoregressive decode step on one CUDA device.  Plain pointers and sizes
 * only; every function returns a status (T2SX_OK == 0) and t2sx_last_error() describes the
 * last failure of the calling thread.  Citations name the reference interface each entry point
 * replaces (include/gpt_sovits/t2s.h and the sources under src/t2s).
 *
 * Threading: a session is a single-owner object (as t2s_session is); different sessions may be
 * driven from different host threads.  All device work of a session runs on its own stream.
 */
#ifndef T2SX_H
#define T2SX_H

#include <stdint.h>

#if defined(__GNUC__)
#define T2SX_API __attribute__((visibility("default")))
#else
#define T2SX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define T2SX_OK 0
#define T2SX_ERR_INVALID 1   /* bad argument / plan (reference: false return or GGML_ASSERT) */
#define T2SX_ERR_IO 2        /* file missing or unreadable (t2s_model_load returns false) */
#define T2SX_ERR_FORMAT 3    /* GGUF malformed, tensor missing or unsupported type */
#define T2SX_ERR_CUDA 4      /* CUDA runtime failure */
#define T2SX_ERR_OOM 5       /* device memory exhausted */
#define T2SX_ERR_STATE 6     /* illegal slot transition (reference aborts via GGML_ASSERT) */
#define T2SX_ERR_BOUNDS 7    /* a slot ran past its capacity (device-side check) */
#define T2SX_ERR_TIMEOUT 8   /* a tensor-core matmul gave up a bounded wait (about 1 s); its outputs are NaN */

typedef struct t2sx_model t2sx_model;
typedef struct t2sx_session t2sx_session;

/* Sampler parameters, bound at session creation (t2s_sampler_config, t2s.h:279-284).
 * eos_mask != 0 sets logit[eos] = -inf after the repetition penalty (not in the reference
 * sampler; used to decode fixed-length sequences). */
typedef struct t2sx_sampler_config {
    int32_t top_k;
    float top_p;
    float temperature;
    float repetition_penalty;
    int32_t eos_mask;
} t2sx_sampler_config;

T2SX_API const char* t2sx_last_error(void);
T2SX_API int t2sx_version(void);
T2SX_API int t2sx_device_count(int32_t* n);

/* t2s_model_load / t2s_model_free (t2s.h:269-272, src/t2s/loader.cpp:140-240): parse the GGUF,
 * read hparams with the reference defaults (loader.cpp:39-50), repack every linear weight into
 * the device layout and upload it to `device`. */
T2SX_API int t2sx_model_load(const char* path, int32_t device, t2sx_model** out);
T2SX_API void t2sx_model_free(t2sx_model* model);
/* hp[9] = embedding_dim, hidden_dim, n_head, linear_units, n_layer, vocab_size,
 * phoneme_vocab_size, eos, inter_channels (t2s_hparams, t2s.h:215-225);
 * wtypes[4] = ggml types of qkv_w, lm_head_w, audio_embedding, bert_proj_w. */
T2SX_API int t2sx_model_hparams(const t2sx_model* model, uint32_t* hp, int32_t* wtypes);
/* Device bytes held by the model's weights. */
T2SX_API int t2sx_model_device_bytes(const t2sx_model* model, uint64_t* bytes);

/* t2s_session_init / t2s_session_free (t2s.h:385-394, session.cpp:55-213).  n_slots concurrent
 * sequences, slot_size positions each; the KV cache is paged f16 (64 positions per page, all
 * layers) sized n_slots * ceil(slot_size / 64) pages.  n_slots == 0 or slot_size == 0 ->
 * T2SX_ERR_INVALID (session.cpp:64-67). */
T2SX_API int t2sx_session_create(const t2sx_model* model, uint32_t n_slots, uint32_t slot_size,
                        const t2sx_sampler_config* cfg, t2sx_session** out);
T2SX_API void t2sx_session_free(t2sx_session* s);
/* t2s_session_find_free_slot (t2s.h:400, session.cpp:215-222): first slot with n_pos == 0, or -1. */
T2SX_API int t2sx_session_find_free_slot(const t2sx_session* s);
/* t2s_session_slot_release (t2s.h:404, session.cpp:224-240). */
T2SX_API int t2sx_session_slot_release(t2sx_session* s, int32_t slot);
/* t2s_session_slot_n_pos (t2s.h:418, session.cpp:242-245); -1 for a bad slot. */
T2SX_API int t2sx_session_slot_n_pos(const t2sx_session* s, int32_t slot);
T2SX_API int t2sx_session_slot_audio_offset(const t2sx_session* s, int32_t slot);
/* Device bytes held by the session (KV pages and work buffers). */
T2SX_API int t2sx_session_device_bytes(const t2sx_session* s, uint64_t* bytes);

/* Prefill input rows for one prompt (t2s_embed_input_forward / t2s_embed_ref_forward text and
 * audio parts, block.cpp:424-511): text rows [0, T_text) from phoneme ids and BERT features
 * (f32 [T_text][1024]) with PE from position 0, then audio rows from prompt semantic ids with PE
 * from position 0.  Inputs are host pointers; x_out (f32 [T_text+T_prompt][d]) is a host
 * pointer, or a device pointer when x_out_on_device != 0. */
T2SX_API int t2sx_embed_prefill(t2sx_session* s, const int32_t* phones, const float* bert, int32_t T_text,
                       const int32_t* sem, int32_t T_prompt, float* x_out, int32_t x_out_on_device);

/* Prompt semantic codes from HuBERT frames (the code extraction of t2s_session_compute_ref_emb,
 * session.cpp:881-1044; sovits_extract_latent_block_forward, block.cpp:140-189): Conv1d(768, 768,
 * kernel 2, stride 2) over the frames plus bias, then the nearest codebook entry,
 * argmax_c(x . E_c - ||E_c||^2 / 2).  hubert: f32 [T][768] (host), T >= 2; codes_out: int32
 * [(T - 2) / 2 + 1] (host). */
T2SX_API int t2sx_extract_latent(t2sx_session* s, const float* hubert, int32_t T, int32_t* codes_out);

/* Prefill of n idle slots in one pass (t2s_session_build_flex_graph + t2s_session_flex_advance
 * with prefill-only plans, session.cpp:461-859): slot[i] receives n_query[i] rows of x (rows of
 * all slots concatenated in the given order, f32 [sum n_query][d]; host pointer, or device
 * pointer when x_on_device != 0).  t_prompt[i] is the slot's ref_T_prompt: rows
 * [0, n_query - t_prompt) are text (bidirectional among text), the rest audio (causal).  Sets
 * n_pos = n_query and audio_offset = n_query - t_prompt; writes each slot's first token (greedy
 * on the last row) to tokens_out[i] (host, may be NULL).  A busy slot, n_query < t_prompt or
 * n_query > slot_size -> T2SX_ERR_STATE / T2SX_ERR_INVALID. */
T2SX_API int t2sx_prefill(t2sx_session* s, int32_t n, const int32_t* slots, const int32_t* n_query,
                 const int32_t* t_prompt, const float* x, int32_t x_on_device, int32_t* tokens_out);

/* Decode (t2s_session_decode_advance + the persistent decode graph, session.cpp:247-396):
 * n_steps steps over every active slot (n_pos > 0); each step embeds the slot's current token,
 * runs the 24 layers and the sampler and feeds the sampled token back, all on the device (one
 * CUDA graph per step).  tokens_out (host, may be NULL) receives [n_steps][n_active] tokens in
 * slot order.  Any active slot reaching slot_size -> T2SX_ERR_BOUNDS before any work. */
T2SX_API int t2sx_decode(t2sx_session* s, int32_t n_steps, int32_t* tokens_out);
/* Enqueue n_steps decode steps without waiting (tokens stay on the device). */
T2SX_API int t2sx_decode_async(t2sx_session* s, int32_t n_steps);
T2SX_API int t2sx_synchronize(t2sx_session* s);
/* One step driven from host buffers, the reference's decode loop shape
 * (test_t2s_infer.cpp:364-421): tokens_in[n_active] are copied to the device, one step runs,
 * tokens_out[n_active] are copied back.  Either pointer may be NULL (device tokens are used /
 * nothing is copied back). */
T2SX_API int t2sx_decode_step_host(t2sx_session* s, const int32_t* tokens_in, int32_t* tokens_out);
/* Active slots in row order (size >= n_slots); returns their count via *n. */
T2SX_API int t2sx_active_slots(t2sx_session* s, int32_t* slots, int32_t* n);
/* Logits f32 [rows][vocab] of the last pass (decode: one row per active slot; prefill: one
 * row per prefilled slot), before the repetition penalty. */
T2SX_API int t2sx_read_logits(t2sx_session* s, float* out, int32_t max_rows, int32_t* rows);
/* One pass over a mixed plan (t2s_session_build_flex_graph + t2s_session_flex_advance +
 * graph compute with decode and prefill slots, session.cpp:461-859): one decode step of the
 * n_dec active slots dec_slots[] with input tokens dec_tokens[], and the prefill of the n_pre idle
 * slots pre_slots[] (n_query, t_prompt and x as in t2sx_prefill; x is host f32
 * [sum n_query][d]), through the layers once.  tokens_out (host, may be NULL) receives n_dec +
 * n_pre tokens: the decode slots' in argument order, then the prefill slots' first tokens.  Noise
 * rows (t2sx_set_exp_noise) follow the same order.  The tokens equal those of
 * t2sx_decode_step_host and t2sx_prefill run separately.  At most 32768 rows per pass; an idle
 * decode slot, a busy prefill slot or a repeated slot -> T2SX_ERR_STATE / T2SX_ERR_INVALID before
 * any device work. */
T2SX_API int t2sx_flex_step(t2sx_session* s, int32_t n_dec, const int32_t* dec_slots, const int32_t* dec_tokens,
                            int32_t n_pre, const int32_t* pre_slots, const int32_t* n_query, const int32_t* t_prompt,
                            const float* x, int32_t* tokens_out);
/* Final-layer output rows f32 [rows][d] of the last pass (the flex graph's y, t2s.h:530): prefill
 * and flex passes give every row of the pass in pass order (flex: the decode rows, then the
 * prefill rows in call order; a prefill of more than 32768 rows keeps its last chunk only),
 * decode steps one row per active slot. */
T2SX_API int t2sx_read_hidden(t2sx_session* s, float* out, int32_t max_rows, int32_t* rows);
/* GGUF type, number of dimensions and ne[4] of a named tensor of the loaded file (the shapes
 * t2s_model_weights exposes, t2s.h:231-243; tests/t2s/test_t2s_loader.cpp:33-92). */
T2SX_API int t2sx_model_tensor_info(const t2sx_model* model, const char* name, int32_t* type, int32_t* n_dims,
                                    int64_t* ne);
/* Cached f16 K (which=0) or V (which=1) of one slot and layer: out [n_pos][d] (uint16 bits),
 * n_pos = t2sx_session_slot_n_pos. */
T2SX_API int t2sx_read_kv(t2sx_session* s, int32_t slot, int32_t layer, int32_t which, uint16_t* out);
/* Seen-token mask used by the repetition penalty (t2s_session_get_seen_mask, t2s.h:487): set
 * one slot's mask (uint8 [vocab], nonzero = seen).  The device marks every sampled token. */
T2SX_API int t2sx_set_seen(t2sx_session* s, int32_t slot, const uint8_t* seen);
/* Stochastic sampling (exp_noise input of the reference sampler, t2s.h:27-28,488): noise holds
 * rows x vocab Exp(1) samples (host), row i used by pass row i (decode: active slots in row order;
 * prefill: slots in call order) and indexed by *sorted* position, as in the reference graph
 * (score = probs_sorted / noise, block.cpp:258-267).  The full chain -- repetition penalty,
 * argsort, top-p, temperature, top-k, softmax, argmax(probs / noise) -- then replaces the greedy
 * pick for every following pass until noise is set again; noise == NULL returns to greedy. */
T2SX_API int t2sx_set_exp_noise(t2sx_session* s, const float* noise, int32_t rows);
/* Greedy (argmax) tokens of the last pass, next to the sampled ones (t2s_session_get_greedy). */
T2SX_API int t2sx_read_greedy(t2sx_session* s, int32_t* out, int32_t max_rows, int32_t* rows);
/* Device time of the last t2sx_decode / t2sx_decode_async batch or t2sx_decode_step_host step
 * (graph execution only, without the host copies), in ms (CUDA events). */
T2SX_API int t2sx_last_decode_ms(t2sx_session* s, float* ms);
/* Kernel nodes in the captured decode-step graph (kernels launched per step). */
T2SX_API int t2sx_decode_graph_kernels(t2sx_session* s, int32_t* n);
/* Average device ms of one launch of each decode-step kernel class, replayed on the state of
 * the last decode step: ms[0] attention (one layer), ms[1..5] matmuls qkv, out, ffn-up,
 * ffn-down, lm_head (with their bias/ReLU epilogues), ms[6] residual+LayerNorm,
 * ms[7] activation quantisation of the 2048-wide FFN rows, ms[8] the attention kernel alone
 * (f32 rows; ms[0] adds the conversion for the out-projection).  ms must hold 9 floats. */
T2SX_API int t2sx_profile_step(t2sx_session* s, int32_t iters, float* ms);

/* ---- kernels on caller-provided device buffers (isolated measurements) ------------------- */

/* A linear weight [N][K] given as ggml block bytes on the host (Q8_0, Q4_0, Q4_K, F16 or F32),
 * repacked to the device layout.  K <= 2048 (the largest T2S contraction, the FFN down
 * projection); larger K returns T2SX_ERR_INVALID. */
typedef struct t2sx_weight t2sx_weight;
T2SX_API int t2sx_weight_create(int32_t device, int32_t ggml_type, const void* host_bytes, int64_t N,
                       int64_t K, t2sx_weight** out);
T2SX_API void t2sx_weight_free(t2sx_weight* w);
/* y[M][N] = x[M][K] . W^T (+ bias[N]) on device pointers, with ggml-CPU semantics (activation
 * rows converted to the weight's dot type).  `stream` is a cudaStream_t (0 = legacy default).
 * Asynchronous: a failure inside the kernels (a tensor-core wait that ran out) is reported by
 * t2sx_weight_sync. */
T2SX_API int t2sx_matmul(t2sx_weight* w, const float* x_dev, int64_t M, const float* bias_dev, float* y_dev,
                void* stream);
/* Waits for `stream` and reports whether a matmul on this weight since the last check gave up a
 * bounded wait (T2SX_ERR_TIMEOUT; its outputs are NaN); clears that state.  The reference has no
 * counterpart (ggml's CPU kernels do not wait on anything). */
T2SX_API int t2sx_weight_sync(t2sx_weight* w, void* stream);
/* Test hook, no counterpart in the reference.  cycles > 0: tensor-core matmuls launched (or
 * graphs captured) from now on first wait on a barrier that nothing completes, and every wait of
 * theirs is bounded by `cycles` clock cycles, so the wait runs out and the error path is taken
 * (outputs NaN, T2SX_ERR_TIMEOUT); 0 restores normal operation with the built-in bound of about
 * one second. */
T2SX_API int t2sx_test_set_tc_wait_cycles(int64_t cycles);

/* No counterpart in the reference (its ggml graphs allocate through the backend).  The same
 * matmul as t2sx_matmul, for callers that cannot allocate device memory at call time -- e.g. a
 * streaming server's synthesis thread, where cudaMalloc may synchronise the device and stall
 * every other stream, or a host application that has pre-reserved the device memory budget.
 * Scratch is a fixed array inside the library (every GPU that loads it holds about 4.5 MiB until
 * exit); M * K must not exceed T2SX_NOALLOC_MAX_ELEMS or the call fails with T2SX_ERR_INVALID.
 * The first call on a device looks up that array's device address (make it before any stream
 * capture).  All calls share the array, so calls that overlap on the GPU race: serialise them. */
#define T2SX_NOALLOC_MAX_ELEMS (1 << 21)
T2SX_API int t2sx_matmul_noalloc(t2sx_weight* w, const float* x_dev, int64_t M, const float* bias_dev,
                                 float* y_dev, void* stream);

/* ---- roofline denominators measured on the device (no counterpart in the reference) ----
 * L2 read bandwidth in GB/s: a zero-filled buffer of `bytes` (1 MiB .. 1 GiB; resident in L2 when
 * it fits) streamed `iters` times with 16-byte loads cached in L2 only, after three warm passes. */
T2SX_API int t2sx_probe_l2_read(int32_t device, int64_t bytes, int32_t iters, double* gbs);
/* Dense int8 tensor-core rate in TOP/s (10^12 integer multiply-adds x 2 per second): every SM
 * issues `iters` x 4 tcgen05.mma.kind::i8 instructions of M = 128, N = 256, K = 32 from shared
 * memory, from `issuers` (1 or 2) threads into separate TMEM accumulators. */
T2SX_API int t2sx_probe_i8_mma(int32_t device, int32_t iters, int32_t issuers, double* tops);

/* ---- isolated batched attention over a paged f16 KV cache (one layer) ----
 * The attention step of t2s_attention_block_forward (src/t2s/block.cpp:575-608) on a stand-alone
 * cache, with the decode and prefill kernels of the step: softmax(q . k^T / sqrt(32)) . v per head
 * over positions [0, len) of a sequence.  The reference has no such entry point (its attention
 * only runs inside the layer graph); this one serves the batched-attention checks and sweep.
 * Calls are ordered on the stream they are given; do not overlap calls on different streams. */
typedef struct t2sx_kvcache t2sx_kvcache;
/* n_seqs sequences of up to max_len positions, pages zero-filled. */
T2SX_API int t2sx_kvcache_create(int32_t device, int32_t n_seqs, int32_t max_len, t2sx_kvcache** out);
T2SX_API void t2sx_kvcache_free(t2sx_kvcache* c);
/* Positions [pos0, pos0 + len) of sequence seq := k, v (host, f16 bits [len][16 heads][32]). */
T2SX_API int t2sx_kvcache_write(t2sx_kvcache* c, int32_t seq, int32_t pos0, int32_t len, const uint16_t* k,
                                const uint16_t* v);
/* Row r (q_dev f16 [n][512]) attends to positions [0, lens[r]) of sequence seqs[r] (host arrays);
 * out_dev f32 [n][512] (32 position lanes per head, butterfly merge).  The two entry points give
 * the same result; the prefill one runs consecutive rows of one sequence (a prompt's rows, each
 * with its own causal prefix length) together, reading their K/V once per 16 rows, as the
 * session prefill does. */
T2SX_API int t2sx_kvcache_attn_decode(t2sx_kvcache* c, int32_t n, const int32_t* seqs, const int32_t* lens,
                                      const uint16_t* q_dev, float* out_dev, void* stream);
T2SX_API int t2sx_kvcache_attn_prefill(t2sx_kvcache* c, int32_t n, const int32_t* seqs, const int32_t* lens,
                                       const uint16_t* q_dev, float* out_dev, void* stream);

#ifdef __cplusplus
}
#endif
#endif
