// Internal interfaces between the engine (engine.cu) and the kernel files.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <string>

namespace sd {

constexpr int kMaxDevices = 64;

// Sets the message sd_last_error() returns on this thread.
void set_last_error(const std::string& s);

// Error codes a kernel writes to its launch's device error word (the first one sticks).
enum : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,   // a consumer gave up waiting for a stage to fill
  kErrTimeoutEmpty = 2,  // a producer gave up waiting for a stage to drain
  kErrTimeoutAccum = 3,  // the epilogue gave up waiting for the accumulator
  kErrBadShape = 4,      // a token id or row index out of range
};

// A block-quantized int4 weight repacked into the GEMM's tile layout (gemm.cu).
struct QWeight {
  uint8_t* tiles = nullptr;
  size_t bytes = 0;
  int n = 0, k = 0, npad = 0;
  bool interleaved = false;
  bool asym = false;     // tiles carry an f16 bias per 32-block: value = q * scale + bias
  int tile_bytes = 0;    // bytes of one 128-row k-tile (codes, scales, and biases when asym)
};

// q, s (and b) in the reference's layout: `bits` (2, 3 or 4) bit codes, one f16 scale (and with b,
// asymmetric weights: one f16 bias) per `group` weights (a multiple of 32); every format becomes the
// int4 tile layout, values unchanged.
cudaError_t repack_weight(const uint8_t* q, const __half* s, int n, int k, bool interleave, QWeight* out, cudaStream_t st,
                          int bits = 4, int group = 32, const __half* b = nullptr);
void gemm_plan(const QWeight& w, int M, int num_sms, int* bn, int* splits, int* kps);
// y[M][ldy] = act[M][K] W^T, or SwiGLU of interleaved gate/up rows into y[M][N/2] when silu; ws is
// the f32 split-K workspace (M * N floats; smaller disables split-K); *nlaunch gets the kernel count.
// With xadd (f32 rows ldy floats apart, n a multiple of 4, no silu): x += f16(act W^T) instead of y.
// algo: 0, the planner's choice (the small-M mma.sync kernel where K is a multiple of 128 and M <= 16,
// or M <= 64 with n <= 4096; else the tcgen05 tiles); 1, the tcgen05 tiles; 2, the small-M kernel (up
// to 256 tokens).
cudaError_t gemm_q4(const QWeight& w, const __half* act, int M, int lda, __half* y, int ldy, bool silu, float* ws,
                    size_t ws_bytes, int* err, int num_sms, cudaStream_t st, int* nlaunch = nullptr, float* xadd = nullptr,
                    int algo = 0);
bool gemm_small_plan(const QWeight& w, int M, int num_sms, int* nt, int* splits, int* kts);
int make_act_map(CUtensorMap* map, const void* ptr, int rows, int cols, int ld, int box_rows);
int make_map_3d(CUtensorMap* map, const void* ptr, int x, int y, int z, long long ystride, long long zstride, int box_y);
// The error words of the standalone calls' kernels (no engine: the C ABI's sd_attention*, sd_gdn):
// read and cleared by sd_op_status.
cudaError_t take_gdn_tc_err(int* code);
cudaError_t take_attn_tc_err(int* code);
int make_map_f32(CUtensorMap* map, const void* ptr, long long rows, int cols, long long ld, int box_rows);

// Model dims the kernels are specialised for (src/kernels.rs:813-835).
struct Dims {
  int d = 2048, inter = 6144;
  int h = 16, dk = 128, dv = 128;  // gated delta
  int hq = 8, hk = 2, hd = 256, rd = 64;
  int C() const { return 2 * h * dk + h * dv; }
};

// kernels.cu
cudaError_t launch_embed_norm(const uint32_t* ids, int l, const uint8_t* eq, const __half* es, int bits, int d, int vocab,
                              const float* w, float* x, __half* h, int* err, cudaStream_t st);
cudaError_t launch_add_norm(float* x, const __half* y, const float* w, int l, int d, bool add, __half* h, cudaStream_t st);
cudaError_t launch_final_norm(float* x, const __half* y, const float* w, const int* rows, int nrows, int l, int d, float* out,
                              int* err, cudaStream_t st);
cudaError_t launch_conv(const __half* big, int stride, const float* conv_w, const __half* hist, int l, int C, __half* qkvc,
                        const int* tstart, const __half* const* hseq, const int* tseq, cudaStream_t st);
cudaError_t launch_hist_update(const __half* big, int stride, __half* hist, int l, int C, cudaStream_t st);
// packed sequences: the conv history after each sequence (its last 3 conv input rows, earlier ones
// from its old history h_in[b], null: zeros) to h_out[b] (null entry: skipped)
cudaError_t launch_hist_pack(const __half* big, int stride, int C, const int* seq_off, const int* seq_len,
                             const __half* const* h_in, __half* const* h_out, int nseq, cudaStream_t st);
// packed sequences: each sequence's keys and values, its prefix (kp[b] / vp[b], [hk][plen[b]][hd]) then
// its own rows (kt / vt, [hk][T][hd] at seq_off[b]), gathered into gk / gv [hk][ktot][hd] at rows
// gofs[b] .. + plen[b] + seq_len[b]. max_rows: the largest plen + len.
cudaError_t launch_kv_gather(const __half* kt, const __half* vt, int T, int hk, int hd, const int* seq_off, const int* seq_len,
                             const int* plen, const __half* const* kp, const __half* const* vp, const int* gofs, int ktot,
                             __half* gk, __half* gv, int nseq, int max_rows, cudaStream_t st);
// packed sequences: each sequence's keys and values, its prefix (kp[b] / vp[b], [hk][plen[b]][hd]) then
// its own rows (kt / vt, [hk][T][hd] at seq_off[b]), to k_out[b] / v_out[b] ([hk][plen + len][hd];
// null entry: skipped). max_rows: the largest plen + len.
cudaError_t launch_kv_pack(const __half* kt, const __half* vt, int T, int hk, int hd, const int* seq_off, const int* seq_len,
                           const int* plen, const __half* const* kp, const __half* const* vp, __half* const* k_out,
                           __half* const* v_out, int nseq, int max_rows, cudaStream_t st);
// gates: beta = sigmoid(b), g = log decay = negA softplus(a + dt_bias), both [l][h]
cudaError_t launch_gdn_gates(const __half* big, int stride, int aoff, int boff, const float* neg_a, const float* dt_bias,
                             int l, int h, float* beta, float* g, cudaStream_t st);
// token-serial gated delta rule (one sequence), decay exp(g) per token as the reference computes it
cudaError_t launch_gdn_recurrent(const float* q, const float* k, int qk_stride, const float* v, int v_stride,
                                 const float* beta, const float* g, float* state, bool load_state, float* o, int l,
                                 int h, cudaStream_t st);
// chunked gated delta rule (gdn.cu) over `batch` sequences: q/k/v f32 or f16 rows (head h at
// h * 128), gates [batch][l][h], state [batch][h][128][128], o [batch][l][h * 128] f32
cudaError_t launch_gdn_chunked(const void* q, const void* k, int qk_stride, const void* v, int v_stride, long long seq_qk,
                               long long seq_v, bool in_f16, const float* beta, const float* g, float* state, bool load_state,
                               float* o, int l, int h, int batch, cudaStream_t st);
// packed sequences (token-major; sequence b at seq_off[b] .. + seq_len[b]), each from states[b] (null
// entry: zeros) to states_out[b] (null table or entry: not stored); one CTA walks a sequence's chunks
cudaError_t launch_gdn_chunked_packed(const __half* q, const __half* k, int qk_stride, const __half* v, int v_stride,
                                      const float* beta, const float* g, const float* const* states, float* const* states_out,
                                      float* o, const int* seq_off, const int* seq_len, int nseq, int h, cudaStream_t st);
// the two-phase scan over packed sequences (long ones): chunk_tab [chunks][2] (first token, tokens),
// chunk0[b] the first chunk of sequence b, order the sequences longest first; scratch holds
// gdn_two_phase_packed_scratch(chunks, h) bytes
size_t gdn_two_phase_packed_scratch(int chunks, int h);
cudaError_t launch_gdn_two_phase_packed(const __half* q, const __half* k, int qk_stride, const __half* v, int v_stride,
                                        const float* beta, const float* g, const float* const* s_in, float* const* s_out,
                                        float* o, const int* seq_off, const int* seq_len, const int* chunk0, const int* order,
                                        const int* chunk_tab, int nseq, int chunks, int h, void* scratch, size_t scratch_bytes,
                                        int num_sms, cudaStream_t st);
// two-phase chunked scan for one long sequence (f16 rows): all chunks' intra-chunk work in parallel,
// then the state scan; `scratch` holds gdn_two_phase_scratch(l, h) bytes of per-chunk records
size_t gdn_two_phase_scratch(int l, int h);
cudaError_t launch_gdn_two_phase(const __half* q, const __half* k, int qk_stride, const __half* v, int v_stride,
                                 const float* beta, const float* g, float* state, bool load_state, float* o, int l, int h,
                                 void* scratch, size_t scratch_bytes, cudaStream_t st);
// gdn_tc.cu: the fused chunked scan on tcgen05 (f16 q/k/v rows, head h at h * 128), one CTA per
// (sequence, head). Packed (seq_off non-null): sequence order[y] (null: y) is tokens seq_off[b] ..
// + seq_len[b], from s_in[b] (null table or entry: zeros) to s_out[b] (null: not stored). Batch:
// `walks / h` sequences of l tokens, sequence b at slab b of the q/k/v maps (seq_qk / seq_v elements
// apart) and tokens b * l .. of beta, g and o; state [b][h][128][128] read when load_state, written
// when store_state. beta, g [token][h]; o [token][h * 128] f32.
struct GdnTcArgs {
  const float *beta = nullptr, *g = nullptr;
  float* o = nullptr;
  int h = 0, l = 0;
  const int *seq_off = nullptr, *seq_len = nullptr, *order = nullptr;
  const float* const* s_in = nullptr;
  float* const* s_out = nullptr;
  float* state = nullptr;
  int load_state = 0, store_state = 1;
  int* err = nullptr;  // a bounded wait that gave up records its code here
};
// rows: the token rows of the q/k/v maps (packed: all packed tokens; batch: l)
cudaError_t launch_gdn_tc(const __half* q, const __half* k, int qk_stride, const __half* v, int v_stride, long long seq_qk,
                          long long seq_v, int rows, const GdnTcArgs& a, int walks, cudaStream_t st);
cudaError_t preload_gdn_tc();
cudaError_t launch_gnorm(const float* o, const __half* big, int stride, int zoff, const float* w, int l, int h, __half* out,
                         cudaStream_t st);
cudaError_t launch_qk_prep(const __half* big, int stride, const float* qw, const float* kw, const float* rope, int l, int p,
                           int lt, const Dims& dm, const int* tpos, __half* q, __half* kc, __half* vc, cudaStream_t st);
// out = x + y (y may be null: out = x)
cudaError_t launch_trace(const float* x, const __half* y, int n, float* out, cudaStream_t st);
// the failure path's self-test: a bounded wait that runs out after limit_ns (see kernels.cu)
cudaError_t launch_wait_probe(int* err, unsigned long long limit_ns, cudaStream_t st);
cudaError_t launch_add_bias(__half* y, const float* bias, int l, int d, cudaStream_t st);

// attn.cu: causal GQA attention with the sigmoid output gate (src/kernels.rs:453-541).
// q [hq][l][hd] (rows for this call), k/v caches [hk][lt][hd] with this call's rows at p..p+l-1,
// gate at gate[t * gstride + goff + h * gstep + d] (null: ungated), out [l][hq * hd].
// Packed mode of the attention kernel: query blocks of several sequences continuing one prefix.
struct AttnPacked {
  const int* blk = nullptr;      // [blocks][2]: sequence, first query (within the sequence) of each block
  const int* seq_off = nullptr;  // first packed token of each sequence
  const int* seq_len = nullptr;
  const __half* kt = nullptr;    // [hk][T][hd] keys and values of the packed tokens
  const __half* vt = nullptr;
  int T = 0;
  // prefixes of their own (one snapshot per sequence): [hk][plen[b]][hd] keys and values of each
  // sequence's prefix; null: every sequence continues the one prefix passed to the launch
  const __half* const* kp = nullptr;
  const __half* const* vp = nullptr;
  const int* plen = nullptr;
};
cudaError_t launch_attention(const __half* q, const __half* k, const __half* v, const __half* gate, int gstride, int goff,
                             int gstep, __half* out, int l, int p, int lt, int hq, int hk, int hd, int splits, float* ws,
                             size_t ws_bytes, cudaStream_t st);
// Key splits launch_attention should use for l queries after p cached keys, and the workspace they need.
cudaError_t launch_attention_packed(const __half* q, const __half* k, const __half* v, const __half* gate, int gstride,
                                    int goff, int gstep, __half* out, int T, int p, int lt, int hq, int hk, int hd,
                                    const AttnPacked& pk, int nblk, int splits, float* ws, size_t ws_bytes, cudaStream_t st);
// attn_tc.cu: the same attention on tcgen05 for query blocks of 128 (head dim 256). Single sequence
// (blk null): l queries after p cached keys, query t at row t of q, keys rows 0 .. p + l - 1. Packed
// (blk non-null): [nblk][2] (sequence, first query, a multiple of 128), sequence b at rows seq_off[b]
// .. + seq_len[b] of q, the keys and out, with no prefix.
struct AttnTcArgs {
  const int* blk = nullptr;
  const int* seq_off = nullptr;
  const int* seq_len = nullptr;
  int l = 0, p = 0, hq = 0, hk = 0;
  int batch = 1;  // single-sequence mode: independent sequences (blockIdx.z), q/k/v/gate/out batch-major
  // packed mode with prefixes (continuations): sequence b's keys are rows kbase_tab[b] .. of the K/V
  // tensors, its plen[b]-row prefix first, and its query i sits at position plen[b] + i (null: rows
  // seq_off[b] .., no prefix)
  const int* kbase_tab = nullptr;
  const int* plen = nullptr;
  const __half* gate = nullptr;
  int gstride = 0, goff = 0, gstep = 0;
  __half* out = nullptr;
  int* err = nullptr;  // a bounded wait that gave up records its code here
};
cudaError_t launch_attention_tc(const __half* q, int qrows, const __half* k, const __half* v, int krows, int krows_valid,
                                const AttnTcArgs& a, int nblk, cudaStream_t st);
cudaError_t preload_attention_tc();
int attention_splits_packed(int nblk, int p, int max_len, int hq, int num_sms);
int attention_splits(int l, int p, int hq, int num_sms);
size_t attention_split_bytes(int l, int hq, int splits);

// The pointer head on the device (head.cu). Question q's rows are row0 .. row0 + nrows - 1 of the
// hidden rows (its options, then its answer row); its nrows - 1 probabilities go to probs[prob0 ..];
// scale = dim^-1/2 / max(temperature, 1e-6).
struct HeadQuestion {
  int row0, nrows, prob0, pad;
  double scale;
};
struct HeadWeights {
  const float *nw = nullptr, *nb = nullptr, *qw = nullptr, *qb = nullptr, *kw = nullptr, *kb = nullptr;
};
// xn [nrows_total][d] and proj [nrows_total][dim] f64 are working memory; unrot (d f64, or null)
// maps a rotated torso's rows back to the head's basis first.
cudaError_t launch_head(const float* hidden, int nrows_total, const HeadQuestion* qs, int nq, int d, int dim,
                        const double* unrot, const HeadWeights& hw, double* xn, double* proj, double* probs,
                        cudaStream_t st);
cudaError_t preload_head();

// The wire format on the device (wire.cu). decode_scales_dev: n rows of g 8-bit scale codes (row r's
// 4-byte header at hdr + r hdr_stride, its codes at codes + r code_stride) to fp16 bits at dst + r
// dst_stride; jmax bounds the rows' j. split_rows_dev: bytes [off, off + len) of n rows of `stride`
// bytes to a dense [n][len] array. Both are stream-ordered.
cudaError_t decode_scales_dev(const uint8_t* hdr, size_t hdr_stride, const uint8_t* codes, size_t code_stride, long long n,
                              int g, int jmax, uint16_t* dst, size_t dst_stride, cudaStream_t st);
cudaError_t split_rows_dev(const uint8_t* src, size_t stride, size_t off, size_t len, long long n, uint8_t* dst,
                           cudaStream_t st);

// Load every kernel of a file on the current device (first-use module loads happen at engine
// creation, not inside a timed forward).
cudaError_t preload_gemm();
cudaError_t preload_attention();
cudaError_t preload_gdn();
cudaError_t preload_kernels();

}  // namespace sd
