// Row-wise and recurrent kernels of the torso: embedding, residual RMSNorm, short conv, gated delta
// rule, gated RMSNorm, q/k RMSNorm + partial RoPE + KV-cache write. Each restates one of the
// reference's WGSL kernels (cited per kernel) with the same rounding points: residual stream and
// recurrent math in f32, f16 where the reference stores f16.
#include "common.cuh"
#include "sd_internal.h"

namespace sd {

// Block-wide sum over 256 threads (8 warps).
__device__ __forceinline__ float block_sum256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; i++) t += red[i];
  return t;
}

__device__ __forceinline__ uint32_t ld32u(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// The unsigned code of element e of block blk in a packed row (src/kernels.rs:63-71).
__device__ __forceinline__ uint32_t code_of(const uint8_t* row, int bits, int blk, int e) {
  const uint8_t* b = row + blk * 4 * bits;
  if (bits == 4) return (ld32u(b + 4 * (e >> 3)) >> (4 * (e & 7))) & 15u;
  uint32_t lo = (ld32u(b + 4 * (e >> 4)) >> (2 * (e & 15))) & 3u;
  if (bits == 3) lo |= ((ld32u(b + 8) >> e) & 1u) << 2;
  return lo;
}

// Hidden sizes the row-wise norm kernels take: a multiple of 64 up to kMaxD (one CTA of 256 threads
// per row, each thread holding NP x 8 elements in registers; NP = ceil(d / 2048)).
constexpr int kMaxD = 8192;

// embed (src/kernels.rs:63-89) fused with layer 0's input RMSNorm (add_norm without the residual
// add, src/kernels.rs:93-120): x[t] = dequant(table[ids[t]]) in f32, h[t] = f16(x * inv * w).
template <int NP>
__global__ void __launch_bounds__(256) embed_norm_kernel(const uint32_t* __restrict__ ids, const uint8_t* __restrict__ eq,
                                                         const __half* __restrict__ es, int bits, int d, int vocab,
                                                         const float* __restrict__ w, float* __restrict__ x,
                                                         __half* __restrict__ h, int* err) {
  grid_dep_wait();
  __shared__ float red[8];
  const int t = blockIdx.x;
  uint32_t id = ids[t];
  if (id >= (uint32_t)vocab) {
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrBadShape);
    id = 0;
  }
  const int nb = d / 32;
  const uint8_t* row = eq + (size_t)id * nb * 4 * bits;
  const float half = (float)(1 << (bits - 1));
  float v[8 * NP];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8 * NP; i++) {
    const int c = threadIdx.x + 256 * i;
    float val = 0.0f;
    if (c < d) {
      const int blk = c >> 5;
      val = ((float)code_of(row, bits, blk, c & 31) - half) * __half2float(es[(size_t)id * nb + blk]);
      x[(size_t)t * d + c] = val;
    }
    v[i] = val;
    ss += val * val;
  }
  const float inv = rsqrtf(block_sum256(ss, red) / (float)d + 1e-6f);
#pragma unroll
  for (int i = 0; i < 8 * NP; i++) {
    const int c = threadIdx.x + 256 * i;
    if (c < d) h[(size_t)t * d + c] = __float2half_rn(v[i] * inv * w[c]);
  }
}

// add_norm (src/kernels.rs:93-120): x += y (when add), h = f16(x * rsqrt(mean(x^2) + 1e-6) * w).
// In pass p thread i owns elements 2048p + 8i .. +7 (16- and 32-byte accesses); a pass past d
// holds zeros.
template <int NP>
__global__ void __launch_bounds__(256) add_norm_kernel(float* __restrict__ x, const __half* __restrict__ y,
                                                       const float* __restrict__ w, int d, int add,
                                                       __half* __restrict__ h) {
  grid_dep_wait();
  __shared__ float red[8];
  const int t = blockIdx.x;
  float* xr = x + (size_t)t * d;
  float v[NP][8];
  float ss = 0.0f;
#pragma unroll
  for (int p = 0; p < NP; p++) {
    const int c0 = 2048 * p + threadIdx.x * 8;
#pragma unroll
    for (int i = 0; i < 8; i++) v[p][i] = 0.0f;
    if (c0 < d) {
      float4 a = *reinterpret_cast<const float4*>(xr + c0), b = *reinterpret_cast<const float4*>(xr + c0 + 4);
      v[p][0] = a.x; v[p][1] = a.y; v[p][2] = a.z; v[p][3] = a.w; v[p][4] = b.x; v[p][5] = b.y; v[p][6] = b.z; v[p][7] = b.w;
      if (add) {
        uint4 yy = *reinterpret_cast<const uint4*>(y + (size_t)t * d + c0);
        const __half2* y2 = reinterpret_cast<const __half2*>(&yy);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          float2 f = __half22float2(y2[i]);
          v[p][2 * i] += f.x;
          v[p][2 * i + 1] += f.y;
        }
        *reinterpret_cast<float4*>(xr + c0) = make_float4(v[p][0], v[p][1], v[p][2], v[p][3]);
        *reinterpret_cast<float4*>(xr + c0 + 4) = make_float4(v[p][4], v[p][5], v[p][6], v[p][7]);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) ss += v[p][i] * v[p][i];
  }
  const float inv = rsqrtf(block_sum256(ss, red) / (float)d + 1e-6f);
#pragma unroll
  for (int p = 0; p < NP; p++) {
    const int c0 = 2048 * p + threadIdx.x * 8;
    if (c0 >= d) continue;
    float4 w0 = *reinterpret_cast<const float4*>(w + c0), w1 = *reinterpret_cast<const float4*>(w + c0 + 4);
    const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    uint4 o;
    __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int i = 0; i < 4; i++)
      o2[i] = __floats2half2_rn(v[p][2 * i] * inv * ww[2 * i], v[p][2 * i + 1] * inv * ww[2 * i + 1]);
    *reinterpret_cast<uint4*>(h + (size_t)t * d + c0) = o;
  }
}

// The final norm (src/kernels.rs:93-120 with add and f32 out, src/engine.rs:519-522): for each
// requested row, x += y (y null: nothing to add, the last matmul added its output already),
// out = x * inv * w in f32.
template <int NP>
__global__ void __launch_bounds__(256) final_norm_kernel(float* __restrict__ x, const __half* __restrict__ y,
                                                         const float* __restrict__ w, const int* __restrict__ rows, int l,
                                                         int d, float* __restrict__ out, int* err) {
  grid_dep_wait();
  __shared__ float red[8];
  const int r = rows[blockIdx.x];
  if (r < 0 || r >= l) {  // rows given on the device are checked here
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrBadShape);
    return;
  }
  float v[8 * NP];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8 * NP; i++) {
    const int c = threadIdx.x + 256 * i;
    float a = 0.0f;
    if (c < d) {
      a = x[(size_t)r * d + c];
      if (y) {
        a += __half2float(y[(size_t)r * d + c]);
        x[(size_t)r * d + c] = a;
      }
    }
    v[i] = a;
    ss += a * a;
  }
  const float inv = rsqrtf(block_sum256(ss, red) / (float)d + 1e-6f);
#pragma unroll
  for (int i = 0; i < 8 * NP; i++) {
    const int c = threadIdx.x + 256 * i;
    if (c < d) out[(size_t)blockIdx.x * d + c] = v[i] * inv * w[c];
  }
}

// conv (src/kernels.rs:152-171): depthwise causal conv (4 taps) over the C = q,k,v channels of the
// in_proj output, then SiLU, f16 out. Each thread owns 4 channels (8-byte loads and stores) and
// kConvT consecutive tokens: it loads the kConvT + 3 input rows up front, so all its loads are in
// flight at once, then computes its outputs from registers (about 70 registers, so 7 CTAs of 128
// threads share an SM and keep enough loads in flight for HBM). A tap before the sequence reads the
// history (the last 3 pre-conv rows before it, `hist` [3][C]). With `tstart` (the first token of each
// token's sequence, for several sequences packed back to back) a tap before its token's sequence
// start reads the history, that sequence's own when `hseq` gives one per sequence (hseq[tseq[t]]; a
// null entry: zeros, a fresh sequence); without it all l tokens are one sequence. The output is
// stored as f16 (the reference keeps f32): the chunked scan that reads it rounds q, k and v to f16
// tensor-core operands anyway, after normalising q and k in f32.
constexpr int kConvT = 8;
__global__ void __launch_bounds__(128) conv_kernel(const __half* __restrict__ big, int stride, const float4* __restrict__ cw,
                                                   const __half* __restrict__ hist, int l, int C, const int* __restrict__ tstart,
                                                   const __half* const* __restrict__ hseq, const int* __restrict__ tseq,
                                                   __half* __restrict__ out) {
  grid_dep_wait();
  const int c4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const int t0 = blockIdx.y * kConvT;
  if (c4 >= C || t0 >= l) return;
  uint2 raw[kConvT + 3];  // input rows t0 - 3 .. t0 + kConvT - 1 (zero outside 0 .. l - 1)
#pragma unroll
  for (int r = 0; r < kConvT + 3; r++) {
    const int t = t0 - 3 + r;
    raw[r] = (t >= 0 && t < l) ? *reinterpret_cast<const uint2*>(big + (size_t)t * stride + c4) : make_uint2(0, 0);
  }
  int tst[kConvT];  // each token's sequence start, loaded with the rows (not one dependent load per token)
#pragma unroll
  for (int i = 0; i < kConvT; i++) tst[i] = tstart && t0 + i < l ? tstart[t0 + i] : 0;
  float w[4][4];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const float4 k = cw[c4 + c];
    w[c][0] = k.x, w[c][1] = k.y, w[c][2] = k.z, w[c][3] = k.w;
  }
#pragma unroll
  for (int i = 0; i < kConvT; i++) {
    const int t = t0 + i;
    if (t >= l) break;
    const int st = tst[i];
    float x[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int tt = t - 3 + j;
      uint2 src = raw[i + j];
      if (tt < st) {  // before the sequence: history row 3 + tt - st
        const __half* hp = hseq ? hseq[tseq[t]] : hist;
        src = hp ? *reinterpret_cast<const uint2*>(hp + (size_t)(3 + tt - st) * C + c4) : make_uint2(0, 0);
      }
      const __half2* h2 = reinterpret_cast<const __half2*>(&src);
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const float2 f = __half22float2(h2[c]);
        x[j][2 * c] = f.x, x[j][2 * c + 1] = f.y;
      }
    }
    uint32_t o[2];
#pragma unroll
    for (int c = 0; c < 4; c += 2) {
      float r[2];
#pragma unroll
      for (int u = 0; u < 2; u++) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; j++) acc += w[c + u][j] * x[j][c + u];
        // SiLU; the fast division (within 2 f32 ulp) is far below the f16 rounding of the output
        r[u] = __fdividef(acc, 1.0f + __expf(-acc));
      }
      const __half2 hv = __floats2half2_rn(r[0], r[1]);
      o[c / 2] = *reinterpret_cast<const uint32_t*>(&hv);
    }
    *reinterpret_cast<uint2*>(out + (size_t)t * C + c4) = make_uint2(o[0], o[1]);
  }
}

// hist_update (src/kernels.rs:173-190): the last 3 pre-conv rows of (old history ++ this call).
__global__ void hist_update_kernel(const __half* __restrict__ big, int stride, __half* __restrict__ hist, int l, int C) {
  grid_dep_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  __half v[3];
#pragma unroll
  for (int r = 0; r < 3; r++) {
    const int src = l - 3 + r;
    v[r] = src >= 0 ? big[(size_t)src * stride + c] : hist[(size_t)(src + 3) * C + c];
  }
#pragma unroll
  for (int r = 0; r < 3; r++) hist[(size_t)r * C + c] = v[r];
}

// hist_update_kernel for packed sequences: grid (channel blocks, sequences).
__global__ void hist_pack_kernel(const __half* __restrict__ big, int stride, int C, const int* __restrict__ seq_off,
                                 const int* __restrict__ seq_len, const __half* const* __restrict__ h_in,
                                 __half* const* __restrict__ h_out) {
  grid_dep_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
  __half* dst = h_out[b];
  if (c >= C || !dst) return;
  const __half* old = h_in ? h_in[b] : nullptr;
  const int off = seq_off[b], l = seq_len[b];
#pragma unroll
  for (int r = 0; r < 3; r++) {
    const int src = l - 3 + r;
    dst[(size_t)r * C + c] = src >= 0 ? big[(size_t)(off + src) * stride + c]
                                      : (old ? old[(size_t)(src + 3) * C + c] : __float2half(0.0f));
  }
}

// A sequence's keys and values into its snapshot: grid (row blocks of 8, kv heads, sequences), a warp
// per row, 16 bytes per lane (head dim 256).
__global__ void kv_pack_kernel(const __half* __restrict__ kt, const __half* __restrict__ vt, int T, int hd,
                               const int* __restrict__ seq_off, const int* __restrict__ seq_len, const int* __restrict__ plen,
                               const __half* const* __restrict__ kp, const __half* const* __restrict__ vp,
                               __half* const* __restrict__ k_out, __half* const* __restrict__ v_out) {
  grid_dep_wait();
  const int b = blockIdx.z, kh = blockIdx.y;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  __half *dk = k_out[b], *dv = v_out[b];
  const int p = plen[b], n = p + seq_len[b];
  if (!dk || row >= n) return;
  const __half *sk, *sv;
  if (row < p) {
    sk = kp[b] + ((size_t)kh * p + row) * hd;
    sv = vp[b] + ((size_t)kh * p + row) * hd;
  } else {
    sk = kt + ((size_t)kh * T + seq_off[b] + row - p) * hd;
    sv = vt + ((size_t)kh * T + seq_off[b] + row - p) * hd;
  }
  const size_t o = ((size_t)kh * n + row) * hd;
  for (int c = lane * 8; c < hd; c += 256) {
    *reinterpret_cast<uint4*>(dk + o + c) = *reinterpret_cast<const uint4*>(sk + c);
    *reinterpret_cast<uint4*>(dv + o + c) = *reinterpret_cast<const uint4*>(sv + c);
  }
}

// kv_pack_kernel into one gathered tensor: sequence b's rows at gofs[b] of every head's ktot rows.
__global__ void kv_gather_kernel(const __half* __restrict__ kt, const __half* __restrict__ vt, int T, int hd,
                                 const int* __restrict__ seq_off, const int* __restrict__ seq_len, const int* __restrict__ plen,
                                 const __half* const* __restrict__ kp, const __half* const* __restrict__ vp,
                                 const int* __restrict__ gofs, int ktot, __half* __restrict__ gk, __half* __restrict__ gv) {
  grid_dep_wait();
  const int b = blockIdx.z, kh = blockIdx.y;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int p = plen[b], n = p + seq_len[b];
  if (row >= n) return;
  const __half *sk, *sv;
  if (row < p) {
    sk = kp[b] + ((size_t)kh * p + row) * hd;
    sv = vp[b] + ((size_t)kh * p + row) * hd;
  } else {
    sk = kt + ((size_t)kh * T + seq_off[b] + row - p) * hd;
    sv = vt + ((size_t)kh * T + seq_off[b] + row - p) * hd;
  }
  const size_t o = ((size_t)kh * ktot + gofs[b] + row) * hd;
  for (int c = lane * 8; c < hd; c += 256) {
    *reinterpret_cast<uint4*>(gk + o + c) = *reinterpret_cast<const uint4*>(sk + c);
    *reinterpret_cast<uint4*>(gv + o + c) = *reinterpret_cast<const uint4*>(sv + c);
  }
}

// The per-token gates of the gated delta rule (src/kernels.rs:289-292): beta = sigmoid(b) and the log
// decay g = negA * softplus(a + dt_bias), softplus(x) = x above 20 (the decay is exp(g)).
__global__ void gdn_gates_kernel(const __half* __restrict__ big, int stride, int aoff, int boff, const float* __restrict__ neg_a,
                                 const float* __restrict__ dtb, int l, int h, float* __restrict__ beta,
                                 float* __restrict__ gl) {
  grid_dep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= l * h) return;
  const int t = i / h, hh = i % h;
  const float a = __half2float(big[(size_t)t * stride + aoff + hh]);
  const float b = __half2float(big[(size_t)t * stride + boff + hh]);
  beta[i] = 1.0f / (1.0f + expf(-b));
  const float x = a + dtb[hh];
  const float sp = x > 20.0f ? x : logf(1.0f + expf(x));
  gl[i] = neg_a[hh] * sp;
}

// Gated delta rule, sequential over tokens (src/kernels.rs:257-302): one CTA per (head, 32 value
// columns); warp w owns 8 columns, lane l key dims 4l..4l+3, so a 128x8 slice of the state lives in
// 32 registers per lane. State [h][128][128] f32: loaded when continuing a prefix, always stored.
__global__ void __launch_bounds__(128) gdn_recurrent_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                            int qk_stride, const float* __restrict__ v, int v_stride,
                                                            const float* __restrict__ beta, const float* __restrict__ gl,
                                                            float* __restrict__ state, int load_state,
                                                            float* __restrict__ o, int l, int h) {
  constexpr int DK = 128, DV = 128;
  const int hh = blockIdx.x / (DV / 32);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dv0 = (blockIdx.x % (DV / 32)) * 32 + warp * 8;
  float4 S[8];
  float* sb = state + (size_t)hh * DK * DV + (size_t)(lane * 4) * DV + dv0;
#pragma unroll
  for (int c = 0; c < 8; c++)
    S[c] = load_state ? make_float4(sb[c], sb[DV + c], sb[2 * DV + c], sb[3 * DV + c]) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float qs = rsqrtf((float)DK);
  for (int t = 0; t < l; t++) {
    const float4 q4 = *reinterpret_cast<const float4*>(q + (size_t)t * qk_stride + hh * DK + lane * 4);
    const float4 k4 = *reinterpret_cast<const float4*>(k + (size_t)t * qk_stride + hh * DK + lane * 4);
    const float sq = warp_sum(q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w);
    const float sk = warp_sum(k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w);
    const float rq = rsqrtf(sq + 1e-6f) * qs, rk = rsqrtf(sk + 1e-6f);
    const float4 qn = make_float4(q4.x * rq, q4.y * rq, q4.z * rq, q4.w * rq);
    const float4 kn = make_float4(k4.x * rk, k4.y * rk, k4.z * rk, k4.w * rk);
    const float dc = expf(gl[(size_t)t * h + hh]), bt = beta[(size_t)t * h + hh];
    const float* vt = v + (size_t)t * v_stride + hh * DV + dv0;
    float mine = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; c++) {
      float4 s = S[c];
      s.x *= dc; s.y *= dc; s.z *= dc; s.w *= dc;
      const float kv = warp_sum(s.x * kn.x + s.y * kn.y + s.z * kn.z + s.w * kn.w);
      const float delta = (vt[c] - kv) * bt;
      s.x += kn.x * delta; s.y += kn.y * delta; s.z += kn.z * delta; s.w += kn.w * delta;
      const float oc = warp_sum(s.x * qn.x + s.y * qn.y + s.z * qn.z + s.w * qn.w);
      if (lane == c) mine = oc;
      S[c] = s;
    }
    if (lane < 8) o[(size_t)t * h * DV + hh * DV + dv0 + lane] = mine;
  }
#pragma unroll
  for (int c = 0; c < 8; c++) {
    sb[c] = S[c].x;
    sb[DV + c] = S[c].y;
    sb[2 * DV + c] = S[c].z;
    sb[3 * DV + c] = S[c].w;
  }
}

// gnorm (src/kernels.rs:377-396): per (token, head) RMSNorm over DV = 128, times w and silu(z),
// z from the in_proj row at zoff; one warp per (token, head).
__global__ void __launch_bounds__(128) gnorm_kernel(const float* __restrict__ o, const __half* __restrict__ big, int stride,
                                                    int zoff, const float* __restrict__ w, int l, int h,
                                                    __half* __restrict__ out) {
  grid_dep_wait();
  constexpr int DV = 128;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= l * h) return;
  const int t = row / h, hh = row % h;
  const int c = lane * 4;  // this lane's 4 consecutive channels
  const float4 v = *reinterpret_cast<const float4*>(o + (size_t)t * h * DV + hh * DV + c);
  const uint2 zz = *reinterpret_cast<const uint2*>(big + (size_t)t * stride + zoff + hh * DV + c);
  const float4 ww = *reinterpret_cast<const float4*>(w + c);
  const float inv = rsqrtf(warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w) / (float)DV + 1e-6f);
  const float2 z01 = __half22float2(*reinterpret_cast<const __half2*>(&zz.x));
  const float2 z23 = __half22float2(*reinterpret_cast<const __half2*>(&zz.y));
  const float vv[4] = {v.x, v.y, v.z, v.w}, wv[4] = {ww.x, ww.y, ww.z, ww.w}, z[4] = {z01.x, z01.y, z23.x, z23.y};
  float r[4];
#pragma unroll
  for (int i = 0; i < 4; i++)  // silu(z): fast division, within 2 f32 ulp, before the f16 rounding
    r[i] = wv[i] * vv[i] * inv * __fdividef(z[i], 1.0f + __expf(-z[i]));
  const __half2 a = __floats2half2_rn(r[0], r[1]), b = __floats2half2_rn(r[2], r[3]);
  uint2 res;
  res.x = *reinterpret_cast<const uint32_t*>(&a);
  res.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(out + (size_t)t * h * DV + hh * DV + c) = res;
}

// qk_prep (src/kernels.rs:400-448): per (token, head slot) RMSNorm over HD times the q or k norm
// weight, rotate-half RoPE on the first RD dims from the f32 table, Q out [HQ][L][HD] f16, K and V
// into the caches [HK][LT][HD] at position p + t. With `tpos` (packed sequences continuing one
// prefix) token t sits at position tpos[t] and its K and V go to row t of [HK][LT][HD] tail buffers.
__global__ void __launch_bounds__(256) qk_prep_kernel(const __half* __restrict__ big, int stride, const float* __restrict__ qw,
                                                      const float* __restrict__ kw, const float2* __restrict__ rope, int l,
                                                      int p, int lt, int hq, int hk, int rd, const int* __restrict__ tpos,
                                                      __half* __restrict__ qo, __half* __restrict__ ko, __half* __restrict__ vo) {
  grid_dep_wait();
  constexpr int HD = 256;
  __shared__ float red[8];
  __shared__ float nv[HD];
  const int t = blockIdx.x, s = blockIdx.y, d = threadIdx.x;
  const bool isq = s < hq;
  const int pos = tpos ? tpos[t] : p + t;  // RoPE position
  const int krow = tpos ? t : pos;         // K/V row
  const __half* row = big + (size_t)t * stride;
  const int koff = hq * HD * 2, voff = koff + hk * HD;
  if (!isq) {
    const int kh = s - hq;
    vo[((size_t)kh * lt + krow) * HD + d] = row[voff + kh * HD + d];
  }
  const float v = __half2float(row[isq ? s * 2 * HD + d : koff + (s - hq) * HD + d]);
  const float tot = block_sum256(v * v, red);
  const float n = v * rsqrtf(tot / (float)HD + 1e-6f) * (isq ? qw[d] : kw[d]);
  nv[d] = n;
  __syncthreads();
  float r = n;
  const int rd2 = rd / 2;
  if (d < rd) {
    const float2 cs = rope[(size_t)pos * rd2 + (d % rd2)];
    r = d < rd2 ? n * cs.x - nv[d + rd2] * cs.y : n * cs.x + nv[d - rd2] * cs.y;
  }
  if (isq) qo[((size_t)s * l + t) * HD + d] = __float2half_rn(r);
  else ko[((size_t)(s - hq) * lt + krow) * HD + d] = __float2half_rn(r);
}

// qk_prep_kernel with one warp per (token, head) row: lane i holds elements 8i .. 8i + 7 (16-byte loads
// and stores), the row's mean square is a warp reduction, and a RoPE partner (d -/+ rd/2) lives rd/16
// lanes away (a shuffle). Needs rd / 2 a multiple of 8. Rows: token-major, (hq + hk) per token.
__global__ void __launch_bounds__(256) qk_prep_warp_kernel(const __half* __restrict__ big, int stride,
                                                           const float* __restrict__ qw, const float* __restrict__ kw,
                                                           const float2* __restrict__ rope, int l, int p, int lt, int hq,
                                                           int hk, int rd, const int* __restrict__ tpos,
                                                           __half* __restrict__ qo, __half* __restrict__ ko,
                                                           __half* __restrict__ vo) {
  grid_dep_wait();
  constexpr int HD = 256;
  const int lane = threadIdx.x & 31;
  const long long rowid = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int heads = hq + hk;
  if (rowid >= (long long)l * heads) return;
  const int t = (int)(rowid / heads), s = (int)(rowid % heads);
  const bool isq = s < hq;
  const int pos = tpos ? tpos[t] : p + t;  // RoPE position
  const int krow = tpos ? t : pos;         // K/V row
  const __half* row = big + (size_t)t * stride;
  const int koff = hq * HD * 2, voff = koff + hk * HD;
  const int d0 = lane * 8;
  if (!isq) {
    const int kh = s - hq;
    *reinterpret_cast<uint4*>(vo + ((size_t)kh * lt + krow) * HD + d0) =
        *reinterpret_cast<const uint4*>(row + voff + kh * HD + d0);
  }
  const uint4 raw = *reinterpret_cast<const uint4*>(row + (isq ? s * 2 * HD : koff + (s - hq) * HD) + d0);
  const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 f = __half22float2(h2[i]);
    v[2 * i] = f.x, v[2 * i + 1] = f.y;
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; i++) ss += v[i] * v[i];
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)HD + 1e-6f);
  const float* w = isq ? qw : kw;
  float n[8];
#pragma unroll
  for (int i = 0; i < 8; i++) n[i] = v[i] * inv * w[d0 + i];
  // RoPE on the first rd elements: partner d + rd/2 (first half) or d - rd/2 (second half)
  const int rd2 = rd / 2, lofs = rd2 / 8;
  const int src = d0 < rd2 ? lane + lofs : (d0 < rd ? lane - lofs : lane);
  float r[8];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float partner = __shfl_sync(0xffffffffu, n[i], src);
    r[i] = n[i];
    if (d0 < rd) {
      const float2 cs = rope[(size_t)pos * rd2 + ((d0 + i) % rd2)];
      r[i] = d0 < rd2 ? n[i] * cs.x - partner * cs.y : n[i] * cs.x + partner * cs.y;
    }
  }
  uint4 out;
  uint32_t* o32 = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const __half2 hv = __floats2half2_rn(r[2 * i], r[2 * i + 1]);
    o32[i] = *reinterpret_cast<const uint32_t*>(&hv);
  }
  if (isq) *reinterpret_cast<uint4*>(qo + ((size_t)s * l + t) * HD + d0) = out;
  else *reinterpret_cast<uint4*>(ko + ((size_t)(s - hq) * lt + krow) * HD + d0) = out;
}

__global__ void trace_kernel(const float* __restrict__ x, const __half* __restrict__ y, int n, float* __restrict__ out) {
  grid_dep_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = y ? x[i] + __half2float(y[i]) : x[i];
}

// add_bias (src/kernels.rs:138-149): y = f16(y + c[j]).
__global__ void add_bias_kernel(__half* __restrict__ y, const float* __restrict__ c, int n, int d) {
  grid_dep_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    y[i] = __float2half_rn(__half2float(y[i]) + c[i % d]);
}

// ---------------------------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------------------------
static int blocks_for(int64_t n, int per) { return (int)std::min<int64_t>((n + per - 1) / per, 65535); }

static bool norm_dim_ok(int d) { return d > 0 && d <= kMaxD && d % 64 == 0; }

cudaError_t launch_embed_norm(const uint32_t* ids, int l, const uint8_t* eq, const __half* es, int bits, int d, int vocab,
                              const float* w, float* x, __half* h, int* err, cudaStream_t st) {
  if (!norm_dim_ok(d)) return cudaErrorInvalidValue;
  switch ((d + 2047) / 2048) {
    case 1: return launch_dependent(embed_norm_kernel<1>, dim3(l), dim3(256), 0, st, ids, eq, es, bits, d, vocab, w, x, h, err);
    case 2: return launch_dependent(embed_norm_kernel<2>, dim3(l), dim3(256), 0, st, ids, eq, es, bits, d, vocab, w, x, h, err);
    case 3: return launch_dependent(embed_norm_kernel<3>, dim3(l), dim3(256), 0, st, ids, eq, es, bits, d, vocab, w, x, h, err);
    default: return launch_dependent(embed_norm_kernel<4>, dim3(l), dim3(256), 0, st, ids, eq, es, bits, d, vocab, w, x, h, err);
  }
}

cudaError_t launch_add_norm(float* x, const __half* y, const float* w, int l, int d, bool add, __half* h, cudaStream_t st) {
  if (!norm_dim_ok(d)) return cudaErrorInvalidValue;
  const int a = add ? 1 : 0;
  switch ((d + 2047) / 2048) {
    case 1: return launch_dependent(add_norm_kernel<1>, dim3(l), dim3(256), 0, st, x, y, w, d, a, h);
    case 2: return launch_dependent(add_norm_kernel<2>, dim3(l), dim3(256), 0, st, x, y, w, d, a, h);
    case 3: return launch_dependent(add_norm_kernel<3>, dim3(l), dim3(256), 0, st, x, y, w, d, a, h);
    default: return launch_dependent(add_norm_kernel<4>, dim3(l), dim3(256), 0, st, x, y, w, d, a, h);
  }
}

cudaError_t launch_final_norm(float* x, const __half* y, const float* w, const int* rows, int nrows, int l, int d, float* out,
                              int* err, cudaStream_t st) {
  if (nrows <= 0) return cudaSuccess;
  if (!norm_dim_ok(d)) return cudaErrorInvalidValue;
  switch ((d + 2047) / 2048) {
    case 1: return launch_dependent(final_norm_kernel<1>, dim3(nrows), dim3(256), 0, st, x, y, w, rows, l, d, out, err);
    case 2: return launch_dependent(final_norm_kernel<2>, dim3(nrows), dim3(256), 0, st, x, y, w, rows, l, d, out, err);
    case 3: return launch_dependent(final_norm_kernel<3>, dim3(nrows), dim3(256), 0, st, x, y, w, rows, l, d, out, err);
    default: return launch_dependent(final_norm_kernel<4>, dim3(nrows), dim3(256), 0, st, x, y, w, rows, l, d, out, err);
  }
}

cudaError_t launch_conv(const __half* big, int stride, const float* conv_w, const __half* hist, int l, int C, __half* qkvc,
                        const int* tstart, const __half* const* hseq, const int* tseq, cudaStream_t st) {
  if (C % 8 || stride % 8 || (hseq && (!tstart || !tseq))) return cudaErrorInvalidValue;
  dim3 grid((C / 4 + 127) / 128, (l + kConvT - 1) / kConvT);
  return launch_dependent(conv_kernel, grid, dim3(128), 0, st, big, stride, reinterpret_cast<const float4*>(conv_w), hist, l, C,
                          tstart, hseq, tseq, qkvc);
}

cudaError_t launch_hist_update(const __half* big, int stride, __half* hist, int l, int C, cudaStream_t st) {
  return launch_dependent(hist_update_kernel, dim3((C + 255) / 256), dim3(256), 0, st, big, stride, hist, l, C);
}

cudaError_t launch_hist_pack(const __half* big, int stride, int C, const int* seq_off, const int* seq_len,
                             const __half* const* h_in, __half* const* h_out, int nseq, cudaStream_t st) {
  if (nseq <= 0 || nseq > 65535 || !h_out) return cudaErrorInvalidValue;
  return launch_dependent(hist_pack_kernel, dim3((C + 255) / 256, nseq), dim3(256), 0, st, big, stride, C, seq_off, seq_len, h_in,
                          h_out);
}

cudaError_t launch_kv_gather(const __half* kt, const __half* vt, int T, int hk, int hd, const int* seq_off, const int* seq_len,
                             const int* plen, const __half* const* kp, const __half* const* vp, const int* gofs, int ktot,
                             __half* gk, __half* gv, int nseq, int max_rows, cudaStream_t st) {
  if (nseq <= 0 || nseq > 65535 || hk <= 0 || hk > 65535 || hd % 8 || max_rows <= 0 || max_rows > ktot) return cudaErrorInvalidValue;
  return launch_dependent(kv_gather_kernel, dim3((max_rows + 7) / 8, hk, nseq), dim3(256), 0, st, kt, vt, T, hd, seq_off, seq_len,
                          plen, kp, vp, gofs, ktot, gk, gv);
}

cudaError_t launch_kv_pack(const __half* kt, const __half* vt, int T, int hk, int hd, const int* seq_off, const int* seq_len,
                           const int* plen, const __half* const* kp, const __half* const* vp, __half* const* k_out,
                           __half* const* v_out, int nseq, int max_rows, cudaStream_t st) {
  if (nseq <= 0 || nseq > 65535 || hk <= 0 || hk > 65535 || hd % 8 || max_rows <= 0 || !k_out || !v_out)
    return cudaErrorInvalidValue;
  return launch_dependent(kv_pack_kernel, dim3((max_rows + 7) / 8, hk, nseq), dim3(256), 0, st, kt, vt, T, hd, seq_off, seq_len,
                          plen, kp, vp, k_out, v_out);
}

cudaError_t launch_gdn_gates(const __half* big, int stride, int aoff, int boff, const float* neg_a, const float* dt_bias,
                             int l, int h, float* beta, float* gl, cudaStream_t st) {
  return launch_dependent(gdn_gates_kernel, dim3(blocks_for((int64_t)l * h, 256)), dim3(256), 0, st, big, stride, aoff, boff, neg_a,
                          dt_bias, l, h, beta, gl);
}

cudaError_t launch_gdn_recurrent(const float* q, const float* k, int qk_stride, const float* v, int v_stride,
                                 const float* beta, const float* gl, float* state, bool load_state, float* o, int l,
                                 int h, cudaStream_t st) {
  gdn_recurrent_kernel<<<h * 4, 128, 0, st>>>(q, k, qk_stride, v, v_stride, beta, gl, state, load_state ? 1 : 0, o, l, h);
  return cudaGetLastError();
}

cudaError_t launch_gnorm(const float* o, const __half* big, int stride, int zoff, const float* w, int l, int h, __half* out,
                         cudaStream_t st) {
  return launch_dependent(gnorm_kernel, dim3((l * h + 3) / 4), dim3(128), 0, st, o, big, stride, zoff, w, l, h, out);
}

cudaError_t launch_qk_prep(const __half* big, int stride, const float* qw, const float* kw, const float* rope, int l, int p,
                           int lt, const Dims& dm, const int* tpos, __half* q, __half* kc, __half* vc, cudaStream_t st) {
  if (dm.hd != 256) return cudaErrorInvalidValue;
  if ((dm.rd / 2) % 8 == 0 && dm.rd <= 256 && stride % 8 == 0) {  // a warp per row
    const long long rows = (long long)l * (dm.hq + dm.hk);
    return launch_dependent(qk_prep_warp_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, st, big, stride, qw, kw,
                            reinterpret_cast<const float2*>(rope), l, p, lt, dm.hq, dm.hk, dm.rd, tpos, q, kc, vc);
  }
  dim3 grid(l, dm.hq + dm.hk);
  return launch_dependent(qk_prep_kernel, grid, dim3(256), 0, st, big, stride, qw, kw, reinterpret_cast<const float2*>(rope), l, p,
                          lt, dm.hq, dm.hk, dm.rd, tpos, q, kc, vc);
}

// A self-test of the kernels' failure path, which no input can reach: warp 0 waits on an mbarrier
// phase that nothing completes, with a short limit, and gives up (the error code into *err, the CTA's
// abort flag set), while warp 1 waits on another such phase with the kernels' full 2 s limit and must
// leave as soon as it sees the abort flag, as every role of the tcgen05 kernels does. Nothing faults
// and nothing is left waiting: the kernel returns and the host reads the code.
__global__ void wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x < 32) mbar_wait_warp_for(&bar[0], 0, &abort_flag, err, kErrTimeoutFull, limit_ns);
  else mbar_wait_warp(&bar[1], 0, &abort_flag, err, kErrTimeoutEmpty);
  __syncthreads();
}

cudaError_t launch_wait_probe(int* err, unsigned long long limit_ns, cudaStream_t st) {
  wait_probe_kernel<<<1, 64, 0, st>>>(err, limit_ns);
  return cudaGetLastError();
}

// Loads the row-wise kernels on the current device (see preload_gemm).
cudaError_t preload_kernels() {
  cudaFuncAttributes a;
  const void* fns[] = {(const void*)embed_norm_kernel<1>, (const void*)embed_norm_kernel<2>, (const void*)embed_norm_kernel<3>,
                       (const void*)embed_norm_kernel<4>, (const void*)add_norm_kernel<1>,   (const void*)add_norm_kernel<2>,
                       (const void*)add_norm_kernel<3>,   (const void*)add_norm_kernel<4>,   (const void*)final_norm_kernel<1>,
                       (const void*)final_norm_kernel<2>, (const void*)final_norm_kernel<3>, (const void*)final_norm_kernel<4>,
                       (const void*)conv_kernel,       (const void*)hist_update_kernel, (const void*)gdn_gates_kernel,
                       (const void*)gdn_recurrent_kernel, (const void*)gnorm_kernel,  (const void*)qk_prep_kernel,
                       (const void*)trace_kernel,      (const void*)add_bias_kernel,    (const void*)hist_pack_kernel,
                       (const void*)kv_pack_kernel,    (const void*)qk_prep_warp_kernel, (const void*)kv_gather_kernel};
  for (const void* f : fns) {
    cudaError_t e = cudaFuncGetAttributes(&a, f);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_trace(const float* x, const __half* y, int n, float* out, cudaStream_t st) {
  return launch_dependent(trace_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, st, x, y, n, out);
}

cudaError_t launch_add_bias(__half* y, const float* bias, int l, int d, cudaStream_t st) {
  return launch_dependent(add_bias_kernel, dim3(blocks_for((int64_t)l * d, 256)), dim3(256), 0, st, y, bias, l * d, d);
}

}  // namespace sd
