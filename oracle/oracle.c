/* CPU oracle: a plain-C restatement of the reference's sequence-mixing forward.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): used by tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg; never by the product. Each function cites the reference file:line it follows.
 * Rounding points follow the WGSL: the residual stream and recurrent math in f32, matmul inputs
 * and outputs rounded to f16 where the reference stores f16 buffers.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define CONTEXT 4096 /* src/engine.rs:16 */

/* ---------------------------------------------------------------------------------------------
 * IEEE binary16 conversions (the `half` crate's f16::from_f32 and WGSL f16(): round to nearest
 * even; restated from the IEEE 754 definition).
 * ------------------------------------------------------------------------------------------- */
uint16_t or_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x38800000u) { /* normal f16 range (or overflow) */
    uint32_t h = (ax - 0x38000000u) >> 13;
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    if (h >= 0x7c00u) h = 0x7c00u;
    return (uint16_t)(sign | h);
  }
  /* subnormal f16: q = value * 2^24 rounded to nearest even */
  uint32_t e = ax >> 23;
  if (e == 0) return (uint16_t)sign; /* f32 subnormals are far below f16's range */
  uint32_t m = (ax & 0x7fffffu) | 0x800000u;
  uint32_t s = 126u - e;
  if (s >= 25u) return (uint16_t)sign;
  uint32_t q = m >> s;
  uint32_t rem = m & ((1u << s) - 1u), half = 1u << (s - 1u);
  if (rem > half || (rem == half && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

float or_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else { /* subnormal: normalise */
      int sh = 0;
      while (!(m & 0x400u)) { m <<= 1; sh++; }
      m &= 0x3ffu;
      x = sign | ((uint32_t)(113 - sh) << 23) | (m << 13);
    }
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static inline float h2f(uint16_t h) { return or_f16_to_f32(h); }
static inline uint16_t f2h(float f) { return or_f32_to_f16(f); }
static inline float rnd16(float f) { return h2f(f2h(f)); }
static inline float inv_sqrt(float x) { return 1.0f / sqrtf(x); }
static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

void or_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ---------------------------------------------------------------------------------------------
 * Block decoding (src/kernels.rs:545-576; embed's element formula src/kernels.rs:63-71).
 * code(): the unsigned code of element e (0..31) of block blk of a row.
 * ------------------------------------------------------------------------------------------- */
static inline uint32_t rd32(const uint8_t* p) {
  uint32_t w;
  memcpy(&w, p, 4);
  return w;
}

static inline uint32_t code_of(const uint8_t* blkp, int bits, int e) {
  if (bits == 4) return (rd32(blkp + 4 * (e / 8)) >> (4 * (e % 8))) & 15u;
  uint32_t lo = (rd32(blkp + 4 * (e / 16)) >> (2 * (e % 16))) & 3u;
  if (bits == 3) lo |= ((rd32(blkp + 8) >> e) & 1u) << 2;
  return lo;
}

/* Row n of w as f32 values: in f32 (the GEMV and embed path) or rounded through f16 arithmetic
 * (the tiled path's `(vec4<f16>(q) - 8.0) * sc`, src/kernels.rs:671-672). */
static void dequant_row(const OrMat* w, int n, float* out, int f16_math) {
  int nb = w->k / 32, bpb = 4 * w->bits; /* bytes per block */
  const uint8_t* row = w->q + (size_t)n * nb * bpb;
  float half = (float)(1 << (w->bits - 1));
  for (int b = 0; b < nb; b++) {
    size_t gi = ((size_t)n * nb + b) / (size_t)(w->group / 32);
    float sc = h2f(w->s[gi]);
    float bi = w->asym ? h2f(w->b[gi]) : 0.0f;
    for (int e = 0; e < 32; e++) {
      float q = (float)code_of(row + (size_t)b * bpb, w->bits, e);
      float v;
      if (w->asym) v = f16_math ? rnd16(rnd16(q * sc) + bi) : q * sc + bi; /* fma in WGSL; close enough */
      else v = f16_math ? rnd16((q - half) * sc) : (q - half) * sc;
      out[b * 32 + e] = v;
    }
  }
}

/* ---------------------------------------------------------------------------------------------
 * Matmuls: Y[m][n] = f16(sum_k A[m][k] W[n][k]).
 * matmul_gemv (src/kernels.rs:590-635): f32 dequant; per output, 8 split-K lanes take blocks
 * s, s+8, ..; each block adds a left-to-right chain of 8 vec4 dots; the 8 lane partials are then
 * summed in lane order.
 * matmul_tiled (src/kernels.rs:640-709): f16 dequant; each output accumulates vec4 dots block by
 * block in K order.
 * ------------------------------------------------------------------------------------------- */
/* Perturbation probe (off by default): with it set, every matmul adds its f32 partial sums in the
 * opposite order (the tiled kernel's K groups from the last; the GEMV's eight split-K lanes from the
 * last). The result differs from the reference only by f32 summation order; the tests use the
 * difference to measure how far the model's f16 activations drift under such a change, the floor
 * below which no implementation that is not bit-identical can agree with the reference. */
static int g_sum_reversed = 0;
void or_set_sum_reversed(int on) { g_sum_reversed = on != 0; }

static inline float dot4(const float* a, const float* b) {
  return a[0] * b[0] + a[1] * b[1] + a[2] * b[2] + a[3] * b[3];
}

static void matmul_gemv(const float* A, int m, const OrMat* w, uint16_t* Y) {
  int N = w->n, K = w->k, nb = K / 32;
#pragma omp parallel
  {
    float* wr = (float*)malloc(sizeof(float) * K);
#pragma omp for schedule(static)
    for (int n = 0; n < N; n++) {
      dequant_row(w, n, wr, 0);
      for (int r = 0; r < m; r++) {
        const float* a = A + (size_t)r * K;
        float tot = 0.0f;
        for (int s0 = 0; s0 < 8; s0++) {
          const int s = g_sum_reversed ? 7 - s0 : s0;
          float acc = 0.0f;
          for (int b = s; b < nb; b += 8) {
            const float* ab = a + b * 32;
            const float* wb = wr + b * 32;
            float c = dot4(ab, wb);
            for (int i = 1; i < 8; i++) c = c + dot4(ab + 4 * i, wb + 4 * i);
            acc += c;
          }
          tot += acc;
        }
        Y[(size_t)r * N + n] = f2h(tot);
      }
    }
    free(wr);
  }
}

static void matmul_tiled(const float* A, int m, const OrMat* w, uint16_t* Y) {
  int N = w->n, K = w->k;
  /* A transposed in groups of 4 (At[k/4][m][4]) so the row loop vectorises */
  float* At = (float*)malloc(sizeof(float) * (size_t)K * m);
  for (int r = 0; r < m; r++)
    for (int k4 = 0; k4 < K / 4; k4++)
      for (int j = 0; j < 4; j++) At[((size_t)k4 * m + r) * 4 + j] = A[(size_t)r * K + 4 * k4 + j];
#pragma omp parallel
  {
    float* wr = (float*)malloc(sizeof(float) * K);
    float* acc = (float*)malloc(sizeof(float) * m);
#pragma omp for schedule(static)
    for (int n = 0; n < N; n++) {
      dequant_row(w, n, wr, 1);
      for (int r = 0; r < m; r++) acc[r] = 0.0f;
      for (int i4 = 0; i4 < K / 4; i4++) {
        const int k4 = g_sum_reversed ? K / 4 - 1 - i4 : i4;
        const float* wk = wr + 4 * k4;
        const float* ak = At + (size_t)k4 * m * 4;
        for (int r = 0; r < m; r++) acc[r] += dot4(ak + 4 * r, wk);
      }
      for (int r = 0; r < m; r++) Y[(size_t)r * N + n] = f2h(acc[r]);
    }
    free(wr);
    free(acc);
  }
  free(At);
}

/* The variant the reference's plan picks for m rows on a GPU without cooperative matrices
 * (src/engine.rs:418-441): GEMV up to 20 rows or for non-default formats / N % 64 != 0. */
static int tiled_for(int m, const OrMat* w) {
  int def = w->bits == 4 && w->group == 32 && !w->asym;
  return m > 20 && def && (w->n % 64) == 0;
}

static void matmul_f32in(const float* A, int m, const OrMat* w, uint16_t* Y, int variant) {
  int tiled = variant == 0 ? tiled_for(m, w) : variant == 2;
  if (tiled) matmul_tiled(A, m, w, Y);
  else matmul_gemv(A, m, w, Y);
}

void or_matmul(const uint16_t* a, int32_t m, const OrMat* w, uint16_t* y, int32_t force_variant) {
  float* A = (float*)malloc(sizeof(float) * (size_t)m * w->k);
  for (size_t i = 0; i < (size_t)m * w->k; i++) A[i] = h2f(a[i]);
  matmul_f32in(A, m, w, y, force_variant);
  free(A);
}

/* ---------------------------------------------------------------------------------------------
 * Gated delta rule (src/kernels.rs:257-302): per token, S <- decay S; kv = S^T kn;
 * delta = (v - kv) beta; S += kn delta^T; o = S^T qn. State [h][dk][dv] f32.
 * ------------------------------------------------------------------------------------------- */
void or_gdn(const float* q, const float* k, int32_t qk_stride, const float* v, int32_t v_stride,
            const float* beta, const float* decay, float* state, int32_t load_state, float* o,
            int32_t l, int32_t H, int32_t dk, int32_t dv) {
  float qs = 1.0f / sqrtf((float)dk);
#pragma omp parallel for schedule(static)
  for (int h = 0; h < H; h++) {
    float* S = state + (size_t)h * dk * dv;
    if (!load_state) memset(S, 0, sizeof(float) * dk * dv);
    float* qn = (float*)malloc(sizeof(float) * dk);
    float* kn = (float*)malloc(sizeof(float) * dk);
    float* kv = (float*)malloc(sizeof(float) * dv);
    for (int t = 0; t < l; t++) {
      const float* qt = q + (size_t)t * qk_stride + h * dk;
      const float* kt = k + (size_t)t * qk_stride + h * dk;
      const float* vt = v + (size_t)t * v_stride + h * dv;
      float sq = 0.0f, sk = 0.0f;
      for (int i = 0; i < dk; i++) { sq += qt[i] * qt[i]; sk += kt[i] * kt[i]; }
      float rq = inv_sqrt(sq + 1e-6f), rk = inv_sqrt(sk + 1e-6f);
      for (int i = 0; i < dk; i++) { qn[i] = qt[i] * rq * qs; kn[i] = kt[i] * rk; }
      float dc = decay[(size_t)t * H + h], bt = beta[(size_t)t * H + h];
      for (int j = 0; j < dv; j++) kv[j] = 0.0f;
      for (int i = 0; i < dk; i++) {
        float* Si = S + (size_t)i * dv;
        for (int j = 0; j < dv; j++) { Si[j] *= dc; kv[j] += Si[j] * kn[i]; }
      }
      for (int j = 0; j < dv; j++) kv[j] = (vt[j] - kv[j]) * bt; /* delta */
      float* ot = o + (size_t)t * H * dv + h * dv;
      for (int j = 0; j < dv; j++) ot[j] = 0.0f;
      for (int i = 0; i < dk; i++) {
        float* Si = S + (size_t)i * dv;
        for (int j = 0; j < dv; j++) { Si[j] += kn[i] * kv[j]; ot[j] += Si[j] * qn[i]; }
      }
    }
    free(qn);
    free(kn);
    free(kv);
  }
}

/* ---------------------------------------------------------------------------------------------
 * Attention (src/kernels.rs:453-541): blocks of 16 queries, keys in chunks of 256 with an online
 * softmax; q pre-scaled by 1/sqrt(hd) and rounded to f16; f32 scores, probabilities and
 * accumulation; output acc / l * sigmoid(gate) rounded to f16.
 * ------------------------------------------------------------------------------------------- */
void or_attn(const uint16_t* Q, const uint16_t* K, const uint16_t* V, const uint16_t* gate,
             int32_t gstride, int32_t goff, int32_t gstep, uint16_t* out,
             int32_t n, int32_t P, int32_t LT, int32_t hq, int32_t hk, int32_t hd) {
  const int BQ = 16, CH = 256;
  float scale = (float)(1.0 / sqrt((double)hd));
  int nblk = (n + BQ - 1) / BQ;
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int h = 0; h < hq; h++) {
    for (int blk = 0; blk < nblk; blk++) {
      int kh = h / (hq / hk);
      int t0 = blk * BQ;
      int nq = n - t0 < BQ ? n - t0 : BQ;
      int tlast = P + t0 + nq - 1;
      float* q = (float*)malloc(sizeof(float) * BQ * hd);
      float* acc = (float*)calloc((size_t)BQ * hd, sizeof(float));
      float* S = (float*)malloc(sizeof(float) * BQ * CH);
      float mrow[16], lrow[16], alpha[16];
      for (int i = 0; i < BQ; i++) {
        for (int d = 0; d < hd; d++)
          q[i * hd + d] = i < nq ? rnd16(h2f(Q[((size_t)h * n + t0 + i) * hd + d]) * scale) : 0.0f;
        mrow[i] = -1e30f;
        lrow[i] = 0.0f;
      }
      for (int j0 = 0; j0 <= tlast; j0 += CH) {
        for (int c = 0; c < CH; c++) {
          int j = j0 + c;
          float s[16];
          for (int i = 0; i < BQ; i++) s[i] = 0.0f;
          if (j <= tlast) {
            const uint16_t* kr = K + ((size_t)kh * LT + j) * hd;
            for (int d4 = 0; d4 < hd / 4; d4++) {
              float kk[4] = {h2f(kr[4 * d4]), h2f(kr[4 * d4 + 1]), h2f(kr[4 * d4 + 2]), h2f(kr[4 * d4 + 3])};
              for (int i = 0; i < BQ; i++) s[i] += dot4(q + i * hd + 4 * d4, kk);
            }
          }
          for (int i = 0; i < BQ; i++) S[i * CH + c] = (j <= P + t0 + i && i < nq) ? s[i] : -1e30f;
        }
        for (int i = 0; i < BQ; i++) {
          float mx = -1e30f;
          for (int c = 0; c < CH; c++) mx = fmaxf(mx, S[i * CH + c]);
          float mnew = fmaxf(mrow[i], mx), sum = 0.0f;
          for (int c = 0; c < CH; c++) {
            float p = expf(S[i * CH + c] - mnew);
            S[i * CH + c] = p;
            sum += p;
          }
          float a = expf(mrow[i] - mnew);
          alpha[i] = a;
          lrow[i] = lrow[i] * a + sum;
          mrow[i] = mnew;
        }
        int jend = j0 + CH < tlast + 1 ? j0 + CH : tlast + 1;
        for (int i = 0; i < BQ; i++)
          for (int d = 0; d < hd; d++) acc[i * hd + d] *= alpha[i];
        for (int jj = j0; jj < jend; jj++) {
          const uint16_t* vr = V + ((size_t)kh * LT + jj) * hd;
          for (int i = 0; i < BQ; i++) {
            float p = S[i * CH + (jj - j0)];
            float* ai = acc + i * hd;
            for (int d = 0; d < hd; d++) ai[d] += p * h2f(vr[d]);
          }
        }
      }
      for (int i = 0; i < nq; i++) {
        int t = t0 + i;
        for (int d = 0; d < hd; d++) {
          float g = gate ? h2f(gate[(size_t)t * gstride + goff + h * gstep + d]) : 0.0f;
          float r = acc[i * hd + d] / lrow[i];
          if (gate) r = r / (1.0f + expf(-g));
          out[(size_t)t * hq * hd + h * hd + d] = f2h(r);
        }
      }
      free(q);
      free(acc);
      free(S);
    }
  }
}

/* ---------------------------------------------------------------------------------------------
 * The engine: buffers, layer loop and snapshots.
 * ------------------------------------------------------------------------------------------- */
struct OrSnapshot {
  int len;
  int n_lin, n_full;
  float** state;     /* per linear layer [H][DK][DV] */
  uint16_t** hist;   /* per linear layer [3][C] */
  uint16_t** k;      /* per full layer [HK][len][HD] */
  uint16_t** v;
};

struct OrEngine {
  OrModel m;
  int C;             /* conv channels 2 h dk + h dv */
  int n_lin, n_full;
  int* slot;         /* layer -> index among its kind */
  float** state;
  uint16_t** hist;
  uint16_t** kc;     /* [HK][CONTEXT][HD] */
  uint16_t** vc;
  float* rope;       /* [CONTEXT][RD/2][2] */
};

OrEngine* or_engine_create(const OrModel* m) {
  OrEngine* e = (OrEngine*)calloc(1, sizeof(OrEngine));
  e->m = *m;
  if (e->m.context <= 0) e->m.context = CONTEXT;
  e->C = 2 * m->h * m->dk + m->h * m->dv;
  e->slot = (int*)calloc(m->n_layers, sizeof(int));
  for (int i = 0; i < m->n_layers; i++) {
    if (m->layers[i].kind == 0) e->slot[i] = e->n_lin++;
    else if (m->layers[i].kind == 1) e->slot[i] = e->n_full++;
  }
  e->state = (float**)calloc(e->n_lin + 1, sizeof(float*));
  e->hist = (uint16_t**)calloc(e->n_lin + 1, sizeof(uint16_t*));
  for (int i = 0; i < e->n_lin; i++) {
    e->state[i] = (float*)calloc((size_t)m->h * m->dk * m->dv, sizeof(float));
    e->hist[i] = (uint16_t*)calloc((size_t)3 * e->C, sizeof(uint16_t));
  }
  e->kc = (uint16_t**)calloc(e->n_full + 1, sizeof(uint16_t*));
  e->vc = (uint16_t**)calloc(e->n_full + 1, sizeof(uint16_t*));
  size_t kv = (size_t)m->hk * e->m.context * m->hd;
  for (int i = 0; i < e->n_full; i++) {
    e->kc[i] = (uint16_t*)calloc(kv, sizeof(uint16_t));
    e->vc[i] = (uint16_t*)calloc(kv, sizeof(uint16_t));
  }
  /* RoPE table in f64, stored f32 (src/engine.rs:259-269) */
  int rd = m->rd;
  e->rope = (float*)malloc(sizeof(float) * (size_t)e->m.context * rd);
  for (int t = 0; t < e->m.context; t++)
    for (int i = 0; i < rd / 2; i++) {
      double a = (double)t / pow(m->rope_theta, (double)(2 * i) / (double)rd);
      e->rope[(size_t)t * rd + 2 * i] = (float)cos(a);
      e->rope[(size_t)t * rd + 2 * i + 1] = (float)sin(a);
    }
  return e;
}

void or_engine_destroy(OrEngine* e) {
  if (!e) return;
  for (int i = 0; i < e->n_lin; i++) { free(e->state[i]); free(e->hist[i]); }
  for (int i = 0; i < e->n_full; i++) { free(e->kc[i]); free(e->vc[i]); }
  free(e->state); free(e->hist); free(e->kc); free(e->vc); free(e->slot); free(e->rope);
  free(e);
}

int32_t or_snapshot_len(const OrSnapshot* s) { return s ? s->len : 0; }

void or_snapshot_free(OrSnapshot* s) {
  if (!s) return;
  for (int i = 0; i < s->n_lin; i++) { free(s->state[i]); free(s->hist[i]); }
  for (int i = 0; i < s->n_full; i++) { free(s->k[i]); free(s->v[i]); }
  free(s->state); free(s->hist); free(s->k); free(s->v);
  free(s);
}

/* embed (src/kernels.rs:63-89) */
static void k_embed(const OrModel* m, const uint32_t* ids, int l, float* x) {
  int d = m->d;
  for (int t = 0; t < l; t++) dequant_row(&m->embed, (int)ids[t], x + (size_t)t * d, 0);
}

/* add_norm (src/kernels.rs:93-120): optional x += y, RMSNorm eps 1e-6 times w. The per-row sum
 * follows the WGSL: 256 thread partials over c = li + 256 i, then 8 subgroup sums in order. */
static void k_add_norm(float* x, const uint16_t* y, const float* w, int d, int row, int add,
                       uint16_t* h16, float* h32, int out_row) {
  float* xr = x + (size_t)row * d;
  int per = d / 256;
  float part[256];
  for (int li = 0; li < 256; li++) {
    float ss = 0.0f;
    for (int i = 0; i < per; i++) {
      int c = li + 256 * i;
      float a = xr[c];
      if (add) { a += h2f(y[(size_t)row * d + c]); xr[c] = a; }
      ss += a * a;
    }
    part[li] = ss;
  }
  float tot = 0.0f;
  for (int sg = 0; sg < 8; sg++) {
    float s = 0.0f;
    for (int lane = 0; lane < 32; lane++) s += part[sg * 32 + lane];
    tot += s;
  }
  float inv = inv_sqrt(tot / (float)d + 1e-6f);
  for (int c = 0; c < d; c++) {
    float v = xr[c] * inv * w[c];
    if (h16) h16[(size_t)out_row * d + c] = f2h(v);
    else h32[(size_t)out_row * d + c] = v;
  }
}

int or_forward(OrEngine* e, const uint32_t* ids, int32_t l, const int32_t* rows, int32_t nrows,
               const OrSnapshot* cache, int32_t keep, OrSnapshot** snap_out, float* hidden, float* trace) {
  const OrModel* m = &e->m;
  int p = cache ? cache->len : 0;
  int LT = m->context;
  if (l <= 0 || p + l > LT) return -1;
  for (int i = 0; i < nrows; i++)
    if (rows[i] < 0 || rows[i] >= l) return -2;
  for (int t = 0; t < l; t++)
    if ((int)ids[t] >= m->vocab) return -3;
  int d = m->d, I = m->inter, H = m->h, DK = m->dk, DV = m->dv, C = e->C;
  int HQ = m->hq, HK = m->hk, HD = m->hd, RD = m->rd;

  /* restore or clear (src/engine.rs:552-571) */
  if (cache) {
    for (int i = 0; i < e->n_lin; i++) {
      memcpy(e->state[i], cache->state[i], sizeof(float) * (size_t)H * DK * DV);
      memcpy(e->hist[i], cache->hist[i], sizeof(uint16_t) * 3 * (size_t)C);
    }
    for (int i = 0; i < e->n_full; i++)
      for (int kh = 0; kh < HK; kh++) {
        memcpy(e->kc[i] + (size_t)kh * LT * HD, cache->k[i] + (size_t)kh * p * HD, sizeof(uint16_t) * (size_t)p * HD);
        memcpy(e->vc[i] + (size_t)kh * LT * HD, cache->v[i] + (size_t)kh * p * HD, sizeof(uint16_t) * (size_t)p * HD);
      }
  } else {
    for (int i = 0; i < e->n_lin; i++) memset(e->hist[i], 0, sizeof(uint16_t) * 3 * (size_t)C);
  }

  size_t maxn = (size_t)2 * I;
  for (int i = 0; i < m->n_layers; i++) {
    const OrLayer* L = &m->layers[i];
    if (L->kind == 0 && (size_t)L->in_proj.n > maxn) maxn = L->in_proj.n;
    if (L->kind == 1 && (size_t)L->qkv.n > maxn) maxn = L->qkv.n;
  }
  float* x = (float*)calloc((size_t)l * d, sizeof(float));
  uint16_t* h = (uint16_t*)calloc((size_t)l * d, 2);
  float* hf = (float*)calloc((size_t)l * (I > d ? I : d), sizeof(float));
  uint16_t* big = (uint16_t*)calloc((size_t)l * maxn, 2);
  uint16_t* mid = (uint16_t*)calloc((size_t)l * I, 2);
  float* qkvc = (float*)calloc((size_t)l * C, sizeof(float));
  float* of = (float*)calloc((size_t)l * H * DV, sizeof(float));
  uint16_t* o = (uint16_t*)calloc((size_t)l * (HQ * HD > H * DV ? HQ * HD : H * DV), 2);
  uint16_t* y = (uint16_t*)calloc((size_t)l * d, 2);
  uint16_t* Qb = (uint16_t*)calloc((size_t)HQ * l * HD, 2);
  float* beta = (float*)calloc((size_t)l * H, sizeof(float));
  float* decay = (float*)calloc((size_t)l * H, sizeof(float));

  k_embed(m, ids, l, x);
#define MATMUL(a16, kk, W, Y)                                              \
  do {                                                                      \
    for (size_t _i = 0; _i < (size_t)l * (kk); _i++) hf[_i] = h2f((a16)[_i]); \
    matmul_f32in(hf, l, (W), (Y), 0);                                       \
  } while (0)

  for (int li = 0; li < m->n_layers; li++) {
    const OrLayer* L = &m->layers[li];
    /* in_norm: adds the previous layer's output y from layer 1 on (src/engine.rs:465) */
#pragma omp parallel for schedule(static)
    for (int t = 0; t < l; t++) k_add_norm(x, y, L->in_norm, d, t, li > 0, h, NULL, t);
    if (L->kind == 2) {
      /* adapter: y = proj(h) + bias (src/engine.rs:466-472, src/kernels.rs:138-149) */
      MATMUL(h, d, &L->proj, y);
      for (int t = 0; t < l; t++)
        for (int c = 0; c < d; c++) y[(size_t)t * d + c] = f2h(h2f(y[(size_t)t * d + c]) + L->bias[c]);
      goto layer_done;
    }
    if (L->kind == 0) {
      int N = L->in_proj.n;
      int slot = e->slot[li];
      MATMUL(h, d, &L->in_proj, big);
      uint16_t* hist = e->hist[slot];
      /* conv + SiLU (src/kernels.rs:152-170) */
#pragma omp parallel for schedule(static)
      for (int t = 0; t < l; t++)
        for (int c = 0; c < C; c++) {
          float s = 0.0f;
          for (int j = 0; j < 4; j++) {
            int tt = t + j - 3;
            float v = tt >= 0 ? h2f(big[(size_t)tt * N + c]) : h2f(hist[(size_t)(tt + 3) * C + c]);
            s += L->conv[c * 4 + j] * v;
          }
          qkvc[(size_t)t * C + c] = s / (1.0f + expf(-s));
        }
      /* hist_update (src/kernels.rs:173-190) */
      for (int c = 0; c < C; c++) {
        uint16_t v[3];
        for (int r = 0; r < 3; r++) {
          int src = l - 3 + r;
          v[r] = src >= 0 ? big[(size_t)src * N + c] : hist[(size_t)(src + 3) * C + c];
        }
        for (int r = 0; r < 3; r++) hist[(size_t)r * C + c] = v[r];
      }
      /* gates (src/kernels.rs:289-292): a_off = C + H DV, b_off = a_off + H (src/engine.rs:480) */
      int aoff = C + H * DV, boff = aoff + H;
      for (int t = 0; t < l; t++)
        for (int hh = 0; hh < H; hh++) {
          float a = h2f(big[(size_t)t * N + aoff + hh]), b = h2f(big[(size_t)t * N + boff + hh]);
          beta[t * H + hh] = 1.0f / (1.0f + expf(-b));
          float xx = a + L->dt_bias[hh];
          float sp = xx > 20.0f ? xx : logf(1.0f + expf(xx));
          decay[t * H + hh] = expf(L->neg_a[hh] * sp);
        }
      or_gdn(qkvc, qkvc + H * DK, C, qkvc + 2 * H * DK, C, beta, decay, e->state[slot], cache != NULL, of, l, H, DK, DV);
      /* gnorm (src/kernels.rs:377-396), z at offset C of the in_proj row */
#pragma omp parallel for schedule(static)
      for (int t = 0; t < l; t++)
        for (int hh = 0; hh < H; hh++) {
          const float* v = of + (size_t)t * H * DV + hh * DV;
          float ss = 0.0f;
          for (int c = 0; c < DV; c++) ss += v[c] * v[c];
          float inv = inv_sqrt(ss / (float)DV + 1e-6f);
          for (int c = 0; c < DV; c++) {
            float z = h2f(big[(size_t)t * N + C + hh * DV + c]);
            o[(size_t)t * H * DV + hh * DV + c] = f2h(L->gnorm[c] * v[c] * inv * z / (1.0f + expf(-z)));
          }
        }
      MATMUL(o, H * DV, &L->out_proj, y);
    } else {
      int N = L->qkv.n;
      int slot = e->slot[li];
      MATMUL(h, d, &L->qkv, big);
      uint16_t* Kc = e->kc[slot];
      uint16_t* Vc = e->vc[slot];
      int koff = HQ * HD * 2, voff = koff + HK * HD, rd2 = RD / 2;
      /* qk_prep (src/kernels.rs:400-448) */
#pragma omp parallel for collapse(2) schedule(static)
      for (int t = 0; t < l; t++)
        for (int s = 0; s < HQ + HK; s++) {
          int isq = s < HQ, pos = p + t;
          float nv[512];
          const uint16_t* row = big + (size_t)t * N;
          if (!isq) {
            int kh = s - HQ;
            for (int dd = 0; dd < HD; dd++) Vc[((size_t)kh * LT + pos) * HD + dd] = row[voff + kh * HD + dd];
          }
          float tot = 0.0f;
          for (int dd = 0; dd < HD; dd++) {
            float v = h2f(row[isq ? s * 2 * HD + dd : koff + (s - HQ) * HD + dd]);
            nv[dd] = v;
            tot += v * v;
          }
          float inv = inv_sqrt(tot / (float)HD + 1e-6f);
          for (int dd = 0; dd < HD; dd++) nv[dd] = nv[dd] * inv * (isq ? L->q_norm[dd] : L->k_norm[dd]);
          for (int dd = 0; dd < HD; dd++) {
            float r = nv[dd];
            if (dd < RD) {
              int ii = dd % rd2;
              float cs = e->rope[(size_t)pos * RD + 2 * ii], sn = e->rope[(size_t)pos * RD + 2 * ii + 1];
              r = dd < rd2 ? nv[dd] * cs - nv[dd + rd2] * sn : nv[dd] * cs + nv[dd - rd2] * sn;
            }
            if (isq) Qb[((size_t)s * l + t) * HD + dd] = f2h(r);
            else Kc[((size_t)(s - HQ) * LT + pos) * HD + dd] = f2h(r);
          }
        }
      /* attention, gate at h * 2 HD + HD of the qkv row (src/kernels.rs:521) */
      or_attn(Qb, Kc, Vc, big, N, HD, 2 * HD, o, l, p, LT, HQ, HK, HD);
      MATMUL(o, HQ * HD, &L->o_proj, y);
    }
    /* post_norm, MLP (src/engine.rs:513-517) */
#pragma omp parallel for schedule(static)
    for (int t = 0; t < l; t++) k_add_norm(x, y, L->post_norm, d, t, 1, h, NULL, t);
    MATMUL(h, d, &L->gate_up, big);
    for (size_t t = 0; t < (size_t)l; t++)
      for (int j = 0; j < I; j++) {
        float gv = h2f(big[t * 2 * I + j]), uv = h2f(big[t * 2 * I + I + j]);
        mid[t * I + j] = f2h(gv / (1.0f + expf(-gv)) * uv);
      }
    MATMUL(mid, I, &L->down, y);
  layer_done:
    if (trace)
      for (size_t i2 = 0; i2 < (size_t)l * d; i2++) trace[(size_t)li * l * d + i2] = x[i2] + h2f(y[i2]);
  }
  /* final norm with the last residual add, gathered rows, f32 out (src/engine.rs:519-522) */
  for (int r = 0; r < nrows; r++) k_add_norm(x, y, m->final_norm, d, rows[r], 1, NULL, hidden, r);
#undef MATMUL

  if (keep && snap_out) { /* src/engine.rs:592-614 */
    int T = p + l;
    OrSnapshot* s = (OrSnapshot*)calloc(1, sizeof(OrSnapshot));
    s->len = T;
    s->n_lin = e->n_lin;
    s->n_full = e->n_full;
    s->state = (float**)calloc(e->n_lin + 1, sizeof(float*));
    s->hist = (uint16_t**)calloc(e->n_lin + 1, sizeof(uint16_t*));
    s->k = (uint16_t**)calloc(e->n_full + 1, sizeof(uint16_t*));
    s->v = (uint16_t**)calloc(e->n_full + 1, sizeof(uint16_t*));
    for (int i = 0; i < e->n_lin; i++) {
      s->state[i] = (float*)malloc(sizeof(float) * (size_t)H * DK * DV);
      memcpy(s->state[i], e->state[i], sizeof(float) * (size_t)H * DK * DV);
      s->hist[i] = (uint16_t*)malloc(sizeof(uint16_t) * 3 * (size_t)C);
      memcpy(s->hist[i], e->hist[i], sizeof(uint16_t) * 3 * (size_t)C);
    }
    for (int i = 0; i < e->n_full; i++) {
      s->k[i] = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)HK * T * HD);
      s->v[i] = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)HK * T * HD);
      for (int kh = 0; kh < HK; kh++) {
        memcpy(s->k[i] + (size_t)kh * T * HD, e->kc[i] + (size_t)kh * LT * HD, sizeof(uint16_t) * (size_t)T * HD);
        memcpy(s->v[i] + (size_t)kh * T * HD, e->vc[i] + (size_t)kh * LT * HD, sizeof(uint16_t) * (size_t)T * HD);
      }
    }
    *snap_out = s;
  }
  free(x); free(h); free(hf); free(big); free(mid); free(qkvc); free(of); free(o); free(y); free(Qb);
  free(beta); free(decay);
  return 0;
}

/* ---------------------------------------------------------------------------------------------
 * Pointer head (src/head.rs:55-77), f64.
 * ------------------------------------------------------------------------------------------- */
static void head_project(const float* x, int d, const float* nw, const float* nb, const float* w,
                         const float* b, int dim, double* out) {
  double mean = 0.0, var = 0.0;
  for (int j = 0; j < d; j++) mean += (double)x[j];
  mean /= d;
  for (int j = 0; j < d; j++) { double t = (double)x[j] - mean; var += t * t; }
  var /= d;
  double r = 1.0 / sqrt(var + 1e-5);
  double* xn = (double*)malloc(sizeof(double) * d);
  for (int j = 0; j < d; j++) xn[j] = ((double)x[j] - mean) * r * (double)nw[j] + (double)nb[j];
  for (int o = 0; o < dim; o++) {
    double s = 0.0;
    for (int j = 0; j < d; j++) s += (double)w[(size_t)o * d + j] * xn[j];
    out[o] = (double)b[o] + s;
  }
  free(xn);
}

void or_head_probs(const float* hidden, int32_t nrows, int32_t d, const float* nw, const float* nb,
                   const float* qw, const float* qb, const float* kw, const float* kb, int32_t dim,
                   double temperature, double* probs) {
  int nopt = nrows - 1;
  double* q = (double*)malloc(sizeof(double) * dim);
  double* k = (double*)malloc(sizeof(double) * dim);
  head_project(hidden + (size_t)nopt * d, d, nw, nb, qw, qb, dim, q);
  double scale = pow((double)dim, -0.5) / (temperature > 1e-6 ? temperature : 1e-6);
  double mx = -1.79769313486231570e308;
  for (int i = 0; i < nopt; i++) {
    head_project(hidden + (size_t)i * d, d, nw, nb, kw, kb, dim, k);
    double s = 0.0;
    for (int o = 0; o < dim; o++) s += k[o] * q[o];
    probs[i] = s * scale;
    if (probs[i] > mx) mx = probs[i];
  }
  double z = 0.0;
  for (int i = 0; i < nopt; i++) { probs[i] = exp(probs[i] - mx); z += probs[i]; }
  for (int i = 0; i < nopt; i++) probs[i] /= z;
  free(q);
  free(k);
}

/* ---------------------------------------------------------------------------------------------
 * 8-bit scale codes (src/model.rs:219-236): a 4-byte header per row (m as fp16 bits, j as u16),
 * then codes sign << 7 | k; |scale| = fp16(f32(m 2^(-k j / 4096))) with the power in f64.
 * ------------------------------------------------------------------------------------------- */
void or_decode_scales(const uint8_t* src, int32_t n, int32_t g, uint16_t* dst) {
  const uint8_t* codes = src + 4 * (size_t)n;
  for (int r = 0; r < n; r++) {
    uint16_t mb = (uint16_t)(src[4 * r] | (src[4 * r + 1] << 8));
    uint16_t j = (uint16_t)(src[4 * r + 2] | (src[4 * r + 3] << 8));
    double mm = (double)h2f(mb);
    for (int i = 0; i < g; i++) {
      uint8_t c = codes[(size_t)r * g + i];
      int k = c & 127;
      uint16_t mag = f2h((float)(mm * pow(2.0, -(double)(k * j) / 4096.0)));
      dst[(size_t)r * g + i] = (uint16_t)(mag | ((uint16_t)(c & 128) << 8));
    }
  }
}
