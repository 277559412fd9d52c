/* CPU oracle for the strands-decider sequence-mixing forward.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference's WGSL kernels
 * (src/kernels.rs) and of its torso layer loop and snapshot semantics (src/engine.rs), used by the
 * tests, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg as the checker. Nothing in
 * the product links, loads or calls it.
 *
 * Parity status: the reference (Rust + WGSL through wgpu) cannot run here (no Rust toolchain, no
 * graphics stack, no model), and its repository holds no golden vectors for the kernels (its engine
 * parity fixtures need the real weights). The kernel restatement is therefore "parity unpinned"
 * against the reference itself; it is cross-checked against an independent numpy restatement
 * (tests/test_oracle.py) and against the reference tests' own invariant (prefix forward equals full
 * forward, tests/engine_parity.rs:59-85). The host-side formats it shares with the product (prompt
 * text, Python float formatting) are pinned against the reference's fixtures.
 */
#ifndef SD_ORACLE_H
#define SD_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint16_t or_f32_to_f16(float f);
float or_f16_to_f32(uint16_t h);

/* A block-quantized matmul weight (src/kernels.rs:6-13): n rows of k values. */
typedef struct {
  const uint8_t* q;   /* packed codes, n rows of k*bits/8 bytes */
  const uint16_t* s;  /* fp16 scales [n][k/group] */
  const uint16_t* b;  /* fp16 biases [n][k/group] when asym, else NULL */
  int32_t n, k, bits, group, asym;
} OrMat;

typedef struct {
  int32_t kind; /* 0 linear_attention, 1 full_attention, 2 adapter */
  const float* in_norm;
  const float* post_norm;
  OrMat in_proj, out_proj;
  const float* conv;      /* [C][4] */
  const float* neg_a;     /* [H] */
  const float* dt_bias;   /* [H] */
  const float* gnorm;     /* [DV] */
  OrMat qkv, o_proj;
  const float* q_norm;    /* [HD] */
  const float* k_norm;    /* [HD] */
  OrMat proj;
  const float* bias;      /* [D] */
  OrMat gate_up, down;
} OrLayer;

typedef struct {
  int32_t d, inter, hq, hk, hd, h, dk, dv, rd, vocab, n_layers, context;
  double rope_theta;
  OrMat embed;            /* vocab rows of d values */
  const float* final_norm;
  const OrLayer* layers;
} OrModel;

typedef struct OrEngine OrEngine;
typedef struct OrSnapshot OrSnapshot;

OrEngine* or_engine_create(const OrModel* m);
void or_engine_destroy(OrEngine* e);
void or_set_threads(int n);
/* Perturbation probe: every matmul adds its f32 partial sums in the opposite order (off by default). */
void or_set_sum_reversed(int on);

/* Engine::forward (src/engine.rs:529-662): returns 0 or a negative error. hidden: [nrows][d] f32.
 * trace (optional): [n_layers][l][d] f32, the residual stream after each layer (x + y). */
int or_forward(OrEngine* e, const uint32_t* ids, int32_t l, const int32_t* rows, int32_t nrows,
               const OrSnapshot* cache, int32_t keep, OrSnapshot** snap_out, float* hidden, float* trace);
int32_t or_snapshot_len(const OrSnapshot* s);
void or_snapshot_free(OrSnapshot* s);

/* Matmul exactly as the reference dispatches it for m rows (src/engine.rs:414-444): the GEMV
 * (f32 dequant) for m <= 20 or a non-default format, else the tiled kernel (f16 dequant). */
void or_matmul(const uint16_t* a, int32_t m, const OrMat* w, uint16_t* y, int32_t force_variant);

/* Isolated causal GQA attention (src/kernels.rs:453-541) over one sequence: q [hq][l][hd] f16,
 * k/v [hk][lt][hd] f16 (rows p..p+l-1 are this call's), gate [l][gstride] f16 at gate_off + h*gstep
 * (NULL: ungated), out [l][hq*hd] f16. */
void or_attn(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* gate,
             int32_t gstride, int32_t goff, int32_t gstep, uint16_t* out,
             int32_t l, int32_t p, int32_t lt, int32_t hq, int32_t hk, int32_t hd);

/* Gated delta rule core (src/kernels.rs:257-302), sequential over tokens, one sequence:
 * q/k [l][qk_stride] f32 at h*dk, v [l][v_stride] f32 at h*dv, beta/decay [l][h], state [h][dk][dv]
 * (in if load_state, always out), o [l][h*dv] f32. */
void or_gdn(const float* q, const float* k, int32_t qk_stride, const float* v, int32_t v_stride,
            const float* beta, const float* decay, float* state, int32_t load_state, float* o,
            int32_t l, int32_t h, int32_t dk, int32_t dv);

/* head.rs probs (src/head.rs:55-77), f64. */
void or_head_probs(const float* hidden, int32_t nrows, int32_t d, const float* nw, const float* nb,
                   const float* qw, const float* qb, const float* kw, const float* kb, int32_t dim,
                   double temperature, double* probs_out);

/* model.rs decode_scales (src/model.rs:219-236): n rows of g codes -> fp16 bits. */
void or_decode_scales(const uint8_t* src, int32_t n, int32_t g, uint16_t* dst);

#ifdef __cplusplus
}
#endif
#endif
