// The pointer head (`Head::probs`, src/head.rs:55-77) on the device, in f64 as the reference computes
// it: per question, LayerNorm (eps 1e-5) of its option rows and its answer row, the k projection of
// the options and the q projection of the answer (f32 weights promoted to f64), scores k_i . q scaled
// by dim^-1/2 / max(temperature, 1e-6), softmax over the options. The sums run in a different order
// from the host's sequential ones (tree reductions), so results agree with the host head to f64
// rounding, not bit for bit.
#include "common.cuh"
#include "sd_internal.h"

namespace sd {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum (or max) over the block's 8 warps; every thread gets the result.
template <bool kMax>
__device__ __forceinline__ double block_reduce_d(double v, double* red) {
  v = kMax ? warp_max_d(v) : warp_sum_d(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double t = red[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; i++) t = kMax ? fmax(t, red[i]) : t + red[i];
  return t;
}

// One row per block: the rotated torso's rows first go back to the head's basis (an unnormalised
// Walsh-Hadamard transform in f32 with the host's butterfly order, so the same f32 values, then the
// per-channel f64 factor rounded to f32, src/engine.rs:652-660); then LayerNorm in f64 into xn.
__global__ void __launch_bounds__(kThreads) head_norm_kernel(const float* __restrict__ hidden, int d,
                                                             const double* __restrict__ unrot,
                                                             const float* __restrict__ nw,
                                                             const float* __restrict__ nb, double* __restrict__ xn) {
  extern __shared__ float srow[];  // d floats when unrot is set
  __shared__ double red[kThreads / 32];
  const float* x = hidden + (size_t)blockIdx.x * d;
  if (unrot) {
    for (int j = threadIdx.x; j < d; j += kThreads) srow[j] = x[j];
    __syncthreads();
    for (int h = 1; h < d; h *= 2) {
      for (int t = threadIdx.x; t < d / 2; t += kThreads) {
        const int j = (t / h) * 2 * h + (t % h);
        const float a = srow[j], b = srow[j + h];
        srow[j] = a + b;
        srow[j + h] = a - b;
      }
      __syncthreads();
    }
    for (int j = threadIdx.x; j < d; j += kThreads) srow[j] = (float)((double)srow[j] * unrot[j]);
    __syncthreads();
    x = srow;
  }
  double s = 0.0;
  for (int j = threadIdx.x; j < d; j += kThreads) s += (double)x[j];
  const double mean = block_reduce_d<false>(s, red) / d;
  double v = 0.0;
  for (int j = threadIdx.x; j < d; j += kThreads) {
    const double c = (double)x[j] - mean;
    v += c * c;
  }
  const double r = 1.0 / sqrt(block_reduce_d<false>(v, red) / d + 1e-5);
  double* out = xn + (size_t)blockIdx.x * d;
  for (int j = threadIdx.x; j < d; j += kThreads) out[j] = ((double)x[j] - mean) * r * (double)nw[j] + (double)nb[j];
}

// Block (8 outputs, question): warp w computes output o = 8 blockIdx.x + w of every row of the
// question, the k projection for the options and the q projection for the answer row. The weight
// row and the question's normalised rows are re-read from L1 across the row loop.
__global__ void __launch_bounds__(kThreads) head_proj_kernel(const double* __restrict__ xn,
                                                             const HeadQuestion* __restrict__ qs, int d, int dim,
                                                             const float* __restrict__ qw, const float* __restrict__ qb,
                                                             const float* __restrict__ kw, const float* __restrict__ kb,
                                                             double* __restrict__ proj) {
  const HeadQuestion q = qs[blockIdx.y];
  const int o = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (o >= dim) return;
  for (int r = 0; r < q.nrows; r++) {
    const bool answer = r == q.nrows - 1;
    const float* w = (answer ? qw : kw) + (size_t)o * d;
    const double* xr = xn + (size_t)(q.row0 + r) * d;
    double s0 = 0.0, s1 = 0.0;
    int j = lane * 4;
    if ((d & 3) == 0) {
      for (; j < d; j += 128) {
        const float4 wv = *reinterpret_cast<const float4*>(w + j);
        const double2 x0 = *reinterpret_cast<const double2*>(xr + j);
        const double2 x1 = *reinterpret_cast<const double2*>(xr + j + 2);
        s0 = fma((double)wv.x, x0.x, s0);
        s1 = fma((double)wv.y, x0.y, s1);
        s0 = fma((double)wv.z, x1.x, s0);
        s1 = fma((double)wv.w, x1.y, s1);
      }
    } else {
      for (j = lane; j < d; j += 32) s0 = fma((double)w[j], xr[j], s0);
    }
    const double s = warp_sum_d(s0 + s1);
    if (lane == 0) proj[(size_t)(q.row0 + r) * dim + o] = (double)(answer ? qb : kb)[o] + s;
  }
}

// One question per block: scores of its options against its answer row, then the softmax, in place
// in probs.
__global__ void __launch_bounds__(kThreads) head_softmax_kernel(const double* __restrict__ proj,
                                                                const HeadQuestion* __restrict__ qs, int dim,
                                                                double* probs) {
  __shared__ double red[kThreads / 32];
  const HeadQuestion q = qs[blockIdx.x];
  const int nopt = q.nrows - 1, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const double* qv = proj + (size_t)(q.row0 + nopt) * dim;
  double* out = probs + q.prob0;
  for (int i = w; i < nopt; i += kThreads / 32) {
    const double* kv = proj + (size_t)(q.row0 + i) * dim;
    double s = 0.0;
    for (int o = lane; o < dim; o += 32) s = fma(kv[o], qv[o], s);
    s = warp_sum_d(s);
    if (lane == 0) out[i] = s * q.scale;
  }
  __syncthreads();
  double m = -1.79769313486231570e308;
  for (int i = threadIdx.x; i < nopt; i += kThreads) m = fmax(m, out[i]);
  m = block_reduce_d<true>(m, red);
  double z = 0.0;
  for (int i = threadIdx.x; i < nopt; i += kThreads) {
    const double e = exp(out[i] - m);
    out[i] = e;
    z += e;
  }
  z = block_reduce_d<false>(z, red);
  for (int i = threadIdx.x; i < nopt; i += kThreads) out[i] /= z;
}

}  // namespace

cudaError_t launch_head(const float* hidden, int nrows_total, const HeadQuestion* qs, int nq, int d, int dim,
                        const double* unrot, const HeadWeights& hw, double* xn, double* proj, double* probs,
                        cudaStream_t st) {
  if (nrows_total <= 0 || nq <= 0) return cudaSuccess;
  const size_t smem = unrot ? (size_t)d * sizeof(float) : 0;
  head_norm_kernel<<<nrows_total, kThreads, smem, st>>>(hidden, d, unrot, hw.nw, hw.nb, xn);
  head_proj_kernel<<<dim3((dim + 7) / 8, nq), kThreads, 0, st>>>(xn, qs, d, dim, hw.qw, hw.qb, hw.kw, hw.kb, proj);
  head_softmax_kernel<<<nq, kThreads, 0, st>>>(proj, qs, dim, probs);
  return cudaGetLastError();
}

cudaError_t preload_head() {
  cudaFuncAttributes a;
  const void* fns[] = {(const void*)head_norm_kernel, (const void*)head_proj_kernel, (const void*)head_softmax_kernel};
  for (const void* f : fns) {
    cudaError_t e = cudaFuncGetAttributes(&a, f);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace sd
