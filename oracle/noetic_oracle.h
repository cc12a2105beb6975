/*
 * noetic_oracle.h -- C entry points of the CPU oracle.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a C++ restatement of the reference's
 * f32 CPU path (the streaming decoder, sampler, prefix scans, batched
 * forward, seeded initialisation and checkpoint reader/writer of noetic).
 * Only the test suite, the smoke check and the CPU-baseline leg of the
 * benchmark may load it, and only as the checker / the timed CPU baseline.
 * The product library never links, loads or calls it.
 *
 * Parity status: the reference is Rust and there is no Rust toolchain in
 * this image, so the reference itself cannot be run.  The oracle is pinned
 * by the reference's own known-answer tests (infer.rs:311-317 zero-nucleus,
 * tensor.rs:371-382 non-finite softmax, tensor.rs:385-388 worker_count) and
 * property tests (scan.rs:269-288 chunked == sequential, selftest.rs:273-299
 * and 675-717 streaming == batched, tests/engine.rs:178-211 reset == fresh).
 * Bit-exact RNG / seeded-init parity has no known-answer vector in the
 * reference and is unpinned beyond line-by-line review.
 */
#ifndef NOETIC_ORACLE_H
#define NOETIC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors model.rs:20-30 LmConfig. */
typedef struct orc_config {
    uint64_t vocab, d_model, n_layer, expand, conv_k, mlp_mult;
    float eps, tau_max;
} orc_config;

/* Mirrors rng.rs:17-22 (xoshiro256++ state plus the cached normal spare). */
typedef struct orc_rng {
    uint64_t s[4];
    float spare;
    uint32_t has_spare;
} orc_rng;

/* Mirrors infer.rs:211-219 SampleCfg. */
typedef struct orc_sample_cfg {
    float temperature;
    uint64_t top_k;
    float top_p;
    float rep_penalty;
    uint64_t rep_window;
    uint32_t greedy;
} orc_sample_cfg;

/* Diagnostics of one sampling decision (not part of the reference API):
 * how close the decision was to flipping, used to classify token
 * mismatches between two implementations as rounding ties. */
typedef struct orc_sample_info {
    uint32_t token;
    uint32_t kept;          /* nucleus size */
    uint32_t used_below;    /* 1 if the rng.below() fallback was taken */
    double draw;            /* draw = f32_unit * total (before walking) */
    double total;           /* f64 sum of kept probabilities */
    double cdf_margin;      /* distance of draw to the nearest CDF edge, / total */
    double cut_margin;      /* min |cumulative - top_p| at the cut and one entry before it */
    double top2_margin;     /* greedy: best - second best logit */
    double order_margin;    /* min relative gap between the chosen probability and its
                               neighbours in the sorted candidates (a swap of two nearly
                               equal probabilities moves the CDF slots of both) */
} orc_sample_info;

const char *orc_last_error(void);

/* ---- rng.rs ---- */
uint64_t orc_splitmix64(uint64_t *state);
void orc_rng_new(orc_rng *r, uint64_t seed);
uint64_t orc_rng_next_u64(orc_rng *r);
float orc_rng_f32_unit(orc_rng *r);
uint64_t orc_rng_below(orc_rng *r, uint64_t n);
float orc_rng_normal(orc_rng *r);

/* ---- tensor.rs ---- */
uint64_t orc_worker_count(uint64_t requested, uint64_t jobs, uint64_t total_work);
void orc_matvec_nt(const float *w, const float *bias, const float *x, float *out,
                   uint64_t dout, uint64_t din, uint64_t threads);
void orc_gemm_nt(const float *a, const float *b, float *c, uint64_t m, uint64_t k,
                 uint64_t n, uint64_t threads);
void orc_rms_norm_vec(const float *x, const float *w, float eps, float *out, uint64_t d);
float orc_sigmoid(float x);
float orc_silu(float x);
void orc_softmax_inplace(float *x, uint64_t n);
uint64_t orc_argmax(const float *x, uint64_t n);

/* ---- scan.rs ---- */
void orc_scan_sequential(const float *a, const float *b, float *h, uint64_t batch,
                         uint64_t t, uint64_t d, uint64_t threads);
void orc_scan_chunked(const float *a, const float *b, float *h, uint64_t batch,
                      uint64_t t, uint64_t d, uint64_t threads);

/* ---- model.rs / nn.rs ---- */
typedef struct orc_model orc_model;
int orc_config_check(const orc_config *cfg);            /* 0 ok, else error */
orc_model *orc_model_new(const orc_config *cfg, orc_rng *rng);  /* Lm::new */
void orc_model_free(orc_model *m);
uint64_t orc_model_tensor_count(const orc_model *m);
const char *orc_model_tensor_name(const orc_model *m, uint64_t i);
uint64_t orc_model_tensor_rank(const orc_model *m, uint64_t i);
uint64_t orc_model_tensor_dim(const orc_model *m, uint64_t i, uint64_t axis);
float *orc_model_tensor_data(orc_model *m, uint64_t i);
uint64_t orc_model_tensor_numel(const orc_model *m, uint64_t i);
void orc_model_set_threads(orc_model *m, uint64_t threads);

/* scan_adjoint (scan.rs:235-260): c_t = g_t + a_{t+1} c_{t+1}, c_T = 0. */
void orc_scan_adjoint(const float *a, const float *g, float *c, uint64_t batch, uint64_t t, uint64_t d);
/* gemm_tn (tensor.rs:156-198): C[m,n] = A[p,m]^T B[p,n], q ascending, zero A skipped. */
void orc_gemm_tn(const float *a, const float *b, float *c, uint64_t p, uint64_t m, uint64_t n);
/* Op::DwConv backward (autograd.rs:1050-1097): accumulates into gx [batch*t*d],
 * gw [k*d], gb [d]; each nullable. */
void orc_dwconv_backward(const float *x, const float *w, const float *go, float *gx, float *gw, float *gb,
                         uint64_t batch, uint64_t t, uint64_t d, uint64_t k);
/* AdamW::step (optim.rs:33-72) for one parameter tensor; t = step counter after
 * the increment.  Returns nonzero (message in orc_last_error) on invalid
 * hyper-parameters or a non-finite gradient / parameter. */
int orc_adamw_step(float *val, const float *grad, float *m, float *v, uint64_t n, float lr, float b1, float b2,
                   float eps, float wd, uint64_t t, int decay);
/* Graph::softmax_ce forward (autograd.rs:579-624): mean cross-entropy in nats
 * over rows whose target is not 0xFFFFFFFF. */
int orc_softmax_ce(const float *logits, uint64_t rows, uint64_t vocab, const uint32_t *targets, float *loss_out);
/* Lm::loss (model.rs:228-234): batched forward, then softmax_ce; logits_out nullable. */
int orc_lm_loss(const orc_model *m, const uint32_t *ids, const uint32_t *targets, uint64_t batch, uint64_t t,
                int scan_policy, float *loss_out, float *logits_out);
/* Batched forward (model.rs:209-226): logits [batch*t, vocab]. */
int orc_lm_logits(const orc_model *m, const uint32_t *ids, uint64_t batch, uint64_t t,
                  int scan_policy, float *logits_out);
/* Batched forward that also returns the decoder state the prompt leaves
 * (per stream: per layer conv ring [k,E] then h [E]; heads per stream). */
int orc_lm_prefill_state(const orc_model *m, const uint32_t *ids, uint64_t batch,
                         uint64_t t, float *state_out, uint32_t *heads_out,
                         float *last_logits_out);

/* ---- infer.rs ---- */
typedef struct orc_state orc_state;
orc_state *orc_state_new(const orc_model *m);
void orc_state_free(orc_state *s);
void orc_state_reset(orc_state *s);
/* Flattened state: per layer conv ring [k,E] followed by h [E]. */
uint64_t orc_state_numel(const orc_state *s);
void orc_state_get(const orc_state *s, float *out, uint32_t *head);
void orc_state_set(orc_state *s, const float *in, uint32_t head);
/* Decoder::step: writes logits [vocab]; returns 0 or -1 on a bad token. */
int orc_step(const orc_model *m, orc_state *s, uint32_t token, float *logits_out);

uint32_t orc_sample_token(float *logits, uint64_t vocab, const orc_sample_cfg *cfg,
                          const uint32_t *history, uint64_t n_history, orc_rng *rng,
                          orc_sample_info *info);

/* cli.rs:470-518 generate() on token ids (no tokenizer): prefill by
 * stepping, then n sampled tokens.  out_tokens[n]. */
int orc_generate(const orc_model *m, const uint32_t *prompt, uint64_t n_prompt, uint64_t n,
                 const orc_sample_cfg *cfg, orc_rng *rng, uint32_t *out_tokens);

/* ---- ckpt.rs ---- */
uint32_t orc_crc32(const uint8_t *data, uint64_t n);
/* Writes every model tensor plus the given metadata (keys[i] -> values[i]). */
int orc_ckpt_save(const orc_model *m, const char *path, const char *const *keys,
                  const char *const *values, uint64_t n_meta);
/* ckpt::load + config from metadata (cmd_gen rules) + apply_exact into a
 * freshly initialised model (rng consumed by the init, as cmd_gen does). */
orc_model *orc_ckpt_load_model(const char *path, orc_rng *rng);

#ifdef __cplusplus
}
#endif
#endif
