// The gated delta rule (the reference's `Gdn` kernels, src/kernels.rs:193-373) as a chunked scan.
//
// Per token (src/kernels.rs:282-297): q^ = q rsqrt(|q|^2 + 1e-6) / sqrt(DK), k^ = k rsqrt(|k|^2 + 1e-6),
// S <- gamma S; delta = beta (v - S^T k^); S += k^ delta^T; o = S^T q^, with gamma = exp(g).
//
// Chunked form over C = 64 tokens from the chunk's entry state S0, with G_i = sum_{j<=i} g_j and
// Gamma_i = exp(G_i):
//   A[i][j] = beta_i exp(G_i - G_j) (k^_i . k^_j) for j < i;  T = (I + A)^-1 (unit lower triangular)
//   W = T diag(beta Gamma) K^,  U = T diag(beta) V,  delta = U - W S0
//   O = diag(Gamma) Q^ S0 + (Q^ K^T o M) delta,  M[i][j] = exp(G_i - G_j) for j <= i
//   S_C = Gamma_C S0 + K^T diag(exp(G_C - G_i)) delta
// which unrolls the recurrence exactly; only the summation order and the f16 rounding of the
// tensor-core operands differ (accumulation is f32; the state is kept in f32).
//
// The value columns of the state are independent in the recurrence, so a CTA takes one head and a
// slice of DVS value columns of one sequence; the intra-chunk products are recomputed per slice.
// The state slice lives in registers as the accumulator of its own update (warp w owns key rows
// 16w..16w+15) with an f16 copy in shared memory as the operand of W S0 and Q^ S0.
#include <mutex>
#include <string>

#include "../../include/sd_b200.h"
#include "common.cuh"
#include "sd_internal.h"

namespace sd {
namespace {

constexpr int CH = 64;        // tokens per chunk
constexpr int DK = 128;       // key (and value) head dim
constexpr int LQK = DK + 8;   // padded row stride (halves) of 128-wide tiles
constexpr int L64 = CH + 8;   // padded row stride (halves) of 64-wide tiles
constexpr int LA = CH + 1;    // row stride (floats) of the f32 64x64 tiles

template <int DVS>
struct GdnSmem {
  static constexpr int LV = DVS + 8;
  __half q[CH * LQK];
  __half k[CH * LQK];
  __half w[CH * LQK];
  __half v[CH * LV];
  __half t1[CH * L64];
  __half t2[CH * L64];
  __half p[CH * L64];
  __half d[CH * LV];
  __half ds[CH * LV];
  __half s[DK * LV];
  float a[CH * LA];
  float x[CH * LA];
  float y[3 * 16 * 17];
  float beta[CH], g[CH], G[CH];
  // the next chunk's raw f16 inputs, prefetched with cp.async while this chunk computes
  __half rq[CH * DK];
  __half rk[CH * DK];
  __half rv[CH * DVS];
  float rbeta[CH], rg[CH];
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t tf32(float x) {  // round to tf32 (nearest, ties away), as the operand
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void mma1688_tf32(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The off-diagonal 16 x 16 blocks of X = (I + A)^-1 (64 x 64, rows LA floats apart, its diagonal blocks
// already solved), level by level: X_ij = -X_ii sum_{m=j}^{i-1} A_im X_mj for i = j + dl; warp w < 4 - dl
// takes block (w + dl, w). The products run on the tensor cores with tf32 operands and f32
// accumulation (tf32 keeps f16's 10-bit mantissa with f32's range: T is rounded to f16 for the W and U
// products right after). `y`: 3 x 16 x 17 floats of scratch. Every thread of the CTA calls it (it
// synchronises the CTA between levels).
__device__ void inverse_offdiag(const float* __restrict__ a, float* __restrict__ x, float* __restrict__ y, int warp, int lane) {
  const int g = lane >> 2, tq = lane & 3;
#pragma unroll 1
  for (int dl = 1; dl < 4; dl++) {
    if (warp < 4 - dl) {
      const int bj = warp, bi = bj + dl;
      float acc[2][4] = {};
      for (int m = bj; m < bi; m++)
#pragma unroll
        for (int kk = 0; kk < 16; kk += 8) {
          const float* ar = a + (bi * 16 + g) * LA + m * 16 + kk;
          const uint32_t a0 = tf32(ar[tq]), a1 = tf32(ar[8 * LA + tq]), a2 = tf32(ar[tq + 4]), a3 = tf32(ar[8 * LA + tq + 4]);
#pragma unroll
          for (int nt = 0; nt < 2; nt++) {
            const float* xr = x + (m * 16 + kk + tq) * LA + bj * 16 + nt * 8 + g;
            mma1688_tf32(acc[nt], a0, a1, a2, a3, tf32(xr[0]), tf32(xr[4 * LA]));
          }
        }
      float* yw = y + warp * 272;  // this block's sum, 16 x 16 (row stride 17)
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        yw[g * 17 + nt * 8 + 2 * tq] = acc[nt][0];
        yw[g * 17 + nt * 8 + 2 * tq + 1] = acc[nt][1];
        yw[(g + 8) * 17 + nt * 8 + 2 * tq] = acc[nt][2];
        yw[(g + 8) * 17 + nt * 8 + 2 * tq + 1] = acc[nt][3];
      }
      __syncwarp();
      float z[2][4] = {};
#pragma unroll
      for (int kk = 0; kk < 16; kk += 8) {
        const float* xr = x + (bi * 16 + g) * LA + bi * 16 + kk;
        const uint32_t a0 = tf32(xr[tq]), a1 = tf32(xr[8 * LA + tq]), a2 = tf32(xr[tq + 4]), a3 = tf32(xr[8 * LA + tq + 4]);
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
          mma1688_tf32(z[nt], a0, a1, a2, a3, tf32(yw[(kk + tq) * 17 + nt * 8 + g]), tf32(yw[(kk + tq + 4) * 17 + nt * 8 + g]));
      }
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        float* xo = x + (bi * 16 + g) * LA + bj * 16 + nt * 8 + 2 * tq;
        xo[0] = -z[nt][0];
        xo[1] = -z[nt][1];
        xo[8 * LA] = -z[nt][2];
        xo[8 * LA + 1] = -z[nt][3];
      }
    }
    __syncthreads();
  }
}

// Fragment addresses (lane-dependent) for the m16n8k16 operands from padded row-major tiles.
// A from [m][k]; B from [n][k] (non-transposed) or [k][n] (transposed); A from [k][m] (transposed).
__device__ __forceinline__ uint32_t a_addr(const __half* base, int ld, int m0, int k0, int lane) {
  const int mat = lane >> 3;
  return smem_u32(base + (m0 + (mat & 1) * 8 + (lane & 7)) * ld + k0 + (mat >> 1) * 8);
}
__device__ __forceinline__ uint32_t bn_addr(const __half* base, int ld, int n0, int k0, int lane) {
  const int mat = lane >> 3;
  return smem_u32(base + (n0 + (mat >> 1) * 8 + (lane & 7)) * ld + k0 + (mat & 1) * 8);
}
__device__ __forceinline__ uint32_t bt_addr(const __half* base, int ld, int k0, int n0, int lane) {
  const int mat = lane >> 3;
  return smem_u32(base + (k0 + (mat & 1) * 8 + (lane & 7)) * ld + n0 + (mat >> 1) * 8);
}
__device__ __forceinline__ uint32_t at_addr(const __half* base, int ld, int k0, int m0, int lane) {
  const int mat = lane >> 3;
  return smem_u32(base + (k0 + (mat >> 1) * 8 + (lane & 7)) * ld + m0 + (mat & 1) * 8);
}

__device__ __forceinline__ void cp_async(void* dst, const void* src, int bytes_valid, int size) {
  if (size == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes_valid) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(bytes_valid) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <typename T>
__device__ __forceinline__ float load1(const T* p) {
  return (float)*p;
}

}  // namespace

template <typename TIn>
struct GdnArgs {
  const TIn *q, *k, *v;
  int qk_stride, v_stride;      // elements between tokens
  long long seq_qk, seq_v;      // elements between sequences
  const float *beta, *g;        // [seq][l][h]
  float* state;                 // [seq][h][128][128]
  float* o;                     // [seq][l][h * 128]
  int load_state, l, h;
  // packed sequences of different lengths (seq_off non-null): sequence b is tokens seq_off[b] ..
  // + seq_len[b] of q, k, v, beta, g and o (token-major, no per-sequence stride)
  const int *seq_off = nullptr, *seq_len = nullptr;
  long long state_bstride = -1;  // elements between sequences' states (-1: h * 128 * 128; 0: one shared state)
  int store_state = 1;           // write the final state back
  // per-sequence states instead of `state` (packed mode): initial states (read only; a null entry:
  // zeros) and where the final ones go (null table or entry: not stored)
  const float* const* states = nullptr;
  float* const* states_out = nullptr;
};

template <int DVS, typename TIn>
__global__ void __launch_bounds__(256, 1) gdn_chunk_kernel(const GdnArgs<TIn> a) {
  constexpr int LV = GdnSmem<DVS>::LV;
  constexpr int NT = DVS / 16;  // n8 tiles per warp for the 64 x DVS products
  extern __shared__ __align__(16) uint8_t gdn_smem_raw[];
  GdnSmem<DVS>& sm = *reinterpret_cast<GdnSmem<DVS>*>(gdn_smem_raw);
  const int NS = DK / DVS;
  const int h = blockIdx.x / NS, c0 = (blockIdx.x % NS) * DVS, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g8 = lane >> 2, tq = lane & 3;
  const int H = a.h;
  const bool packed = a.seq_off != nullptr;
  const long long t_base = packed ? a.seq_off[b] : (long long)b * a.l;  // first token (in beta, g, o)
  const int L = packed ? a.seq_len[b] : a.l;
  const TIn* qg = a.q + (packed ? t_base * a.qk_stride : b * a.seq_qk) + h * DK;
  const TIn* kg = a.k + (packed ? t_base * a.qk_stride : b * a.seq_qk) + h * DK;
  const TIn* vg = a.v + (packed ? t_base * a.v_stride : b * a.seq_v) + h * DK + c0;
  const float* betag = a.beta + t_base * H + h;
  const float* gg = a.g + t_base * H + h;
  float* og = a.o + t_base * H * DK + h * DK + c0;
  const long long sb = a.state_bstride < 0 ? (long long)H * DK * DK : a.state_bstride;
  const long long hoff = (long long)h * DK * DK + c0;
  const float* sin = a.states ? (a.states[b] ? a.states[b] + hoff : nullptr) : (a.load_state ? a.state + b * sb + hoff : nullptr);
  float* sout = a.states ? (a.states_out && a.states_out[b] ? a.states_out[b] + hoff : nullptr)
                         : (a.store_state ? a.state + b * sb + hoff : nullptr);

  // State slice: warp w owns key rows 16w..16w+15, all DVS columns (m16n8 accumulator layout).
  float sacc[DVS / 8][4];
#pragma unroll
  for (int nt = 0; nt < DVS / 8; nt++)
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int row = warp * 16 + g8 + (r >> 1) * 8, col = nt * 8 + 2 * tq + (r & 1);
      sacc[nt][r] = sin ? sin[row * DK + col] : 0.0f;
    }
  auto write_state_f16 = [&]() {
#pragma unroll
    for (int nt = 0; nt < DVS / 8; nt++) {
      const int row = warp * 16 + g8, col = nt * 8 + 2 * tq;
      *reinterpret_cast<__half2*>(&sm.s[row * LV + col]) = __floats2half2_rn(sacc[nt][0], sacc[nt][1]);
      *reinterpret_cast<__half2*>(&sm.s[(row + 8) * LV + col]) = __floats2half2_rn(sacc[nt][2], sacc[nt][3]);
    }
  };
  write_state_f16();

  const float qscale = rsqrtf((float)DK);
  const int mt = warp & 3;             // m16 tile of the 64-row products
  const int nbase = (warp >> 2) * (DVS / 2);  // first value column of this warp's 64 x DVS products

  // f16 inputs are prefetched one chunk ahead into the staging buffers; f32 inputs are read directly
  constexpr bool kStage = sizeof(TIn) == 2;
  auto prefetch = [&](int t0) {
    const int n = min(CH, L - t0);
    for (int e = threadIdx.x; e < CH * (DK / 8); e += 256) {  // q, k: 16 chunks of 16 bytes per row
      const int r = e >> 4, c = (e & 15) * 8;
      const int rr = r < n ? r : 0;
      cp_async(&sm.rq[r * DK + c], qg + (long long)(t0 + rr) * a.qk_stride + c, r < n ? 16 : 0, 16);
      cp_async(&sm.rk[r * DK + c], kg + (long long)(t0 + rr) * a.qk_stride + c, r < n ? 16 : 0, 16);
    }
    for (int e = threadIdx.x; e < CH * (DVS / 8); e += 256) {
      const int r = e / (DVS / 8), c = (e % (DVS / 8)) * 8;
      const int rr = r < n ? r : 0;
      cp_async(&sm.rv[r * DVS + c], vg + (long long)(t0 + rr) * a.v_stride + c, r < n ? 16 : 0, 16);
    }
    if (threadIdx.x < 2 * CH) {
      const int r = threadIdx.x & (CH - 1), rr = r < n ? r : 0;
      const bool isb = threadIdx.x < CH;
      cp_async(isb ? &sm.rbeta[r] : &sm.rg[r], (isb ? betag : gg) + (long long)(t0 + rr) * H, r < n ? 4 : 0, 4);
    }
    cp_async_commit();
  };
  if constexpr (kStage) prefetch(0);

  for (int t0 = 0; t0 < L; t0 += CH) {
    const int n = min(CH, L - t0);
    // 1. normalised q^, k^ (one warp per token row), the value slice, the gates
    if constexpr (kStage) {
      cp_async_wait_all();
      __syncthreads();
    }
    for (int r = warp; r < CH; r += 8) {
      float4 qv = make_float4(0.f, 0.f, 0.f, 0.f), kv = qv;
      if constexpr (kStage) {
        qv = load4<__half>(&sm.rq[r * DK + lane * 4]);
        kv = load4<__half>(&sm.rk[r * DK + lane * 4]);
      } else if (r < n) {
        qv = load4(qg + (long long)(t0 + r) * a.qk_stride + lane * 4);
        kv = load4(kg + (long long)(t0 + r) * a.qk_stride + lane * 4);
      }
      const float sq = warp_sum(qv.x * qv.x + qv.y * qv.y + qv.z * qv.z + qv.w * qv.w);
      const float sk = warp_sum(kv.x * kv.x + kv.y * kv.y + kv.z * kv.z + kv.w * kv.w);
      const float rq = rsqrtf(sq + 1e-6f) * qscale, rk = rsqrtf(sk + 1e-6f);
      __half2* qd = reinterpret_cast<__half2*>(&sm.q[r * LQK + lane * 4]);
      __half2* kd = reinterpret_cast<__half2*>(&sm.k[r * LQK + lane * 4]);
      qd[0] = __floats2half2_rn(qv.x * rq, qv.y * rq);
      qd[1] = __floats2half2_rn(qv.z * rq, qv.w * rq);
      kd[0] = __floats2half2_rn(kv.x * rk, kv.y * rk);
      kd[1] = __floats2half2_rn(kv.z * rk, kv.w * rk);
      for (int j = lane; j < DVS; j += 32) {
        if constexpr (kStage) sm.v[r * LV + j] = sm.rv[r * DVS + j];
        else sm.v[r * LV + j] = __float2half_rn(r < n ? load1(vg + (long long)(t0 + r) * a.v_stride + j) : 0.0f);
      }
    }
    if (threadIdx.x < CH) {
      const int r = threadIdx.x;
      if constexpr (kStage) {
        sm.beta[r] = sm.rbeta[r];
        sm.g[r] = sm.rg[r];
      } else {
        sm.beta[r] = r < n ? betag[(long long)(t0 + r) * H] : 0.0f;
        sm.g[r] = r < n ? gg[(long long)(t0 + r) * H] : 0.0f;
      }
    }
    __syncthreads();
    if constexpr (kStage) {
      if (t0 + CH < L) prefetch(t0 + CH);  // the staging buffers are free again
    }
    if (warp == 0) {  // inclusive prefix sum of the log decays
      const float x0 = sm.g[2 * lane], x1 = sm.g[2 * lane + 1];
      float s = x0 + x1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += u;
      }
      const float before = s - (x0 + x1);
      sm.G[2 * lane] = before + x0;
      sm.G[2 * lane + 1] = s;
    }
    __syncthreads();

    // 2. K^ K^T -> A (masked, scaled, f32) and Q^ K^T -> P (masked, decayed, f16)
    {
      const int nb = (warp >> 2) * 32;
      float kk[4][4], qk[4][4];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) kk[i][j] = qk[i][j] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < DK / 16; ks++) {
        uint32_t ak[4], aq[4];
        ldsm_x4(a_addr(sm.k, LQK, mt * 16, ks * 16, lane), ak);
        ldsm_x4(a_addr(sm.q, LQK, mt * 16, ks * 16, lane), aq);
#pragma unroll
        for (int j2 = 0; j2 < 2; j2++) {
          uint32_t bk[4];
          ldsm_x4(bn_addr(sm.k, LQK, nb + j2 * 16, ks * 16, lane), bk);
          mma16816(kk[2 * j2], ak, bk[0], bk[1]);
          mma16816(kk[2 * j2 + 1], ak, bk[2], bk[3]);
          mma16816(qk[2 * j2], aq, bk[0], bk[1]);
          mma16816(qk[2 * j2 + 1], aq, bk[2], bk[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; nt++)
#pragma unroll
        for (int r = 0; r < 4; r++) {
          const int i = mt * 16 + g8 + (r >> 1) * 8, j = nb + nt * 8 + 2 * tq + (r & 1);
          const float e = j <= i ? __expf(sm.G[i] - sm.G[j]) : 0.0f;
          sm.a[i * LA + j] = j < i ? sm.beta[i] * e * kk[nt][r] : 0.0f;
          sm.p[i * L64 + j] = __float2half_rn(e * qk[nt][r]);
        }
    }
    __syncthreads();

    // 3. T = (I + A)^-1, blocked by 16: diagonal blocks by forward substitution (warp bb, lane =
    // column), then the off-diagonal blocks level by level: X_ij = -X_ii sum_{m=j}^{i-1} A_im X_mj.
    if (warp < 4 && lane < 16) {
      const int o = warp * 16, c = lane;
      float xc[16];
#pragma unroll
      for (int r = 0; r < 16; r++) {
        float val = r == c ? 1.0f : 0.0f;
#pragma unroll
        for (int j = 0; j < r; j++)
          if (j >= c) val -= sm.a[(o + r) * LA + o + j] * xc[j];
        xc[r] = r >= c ? val : 0.0f;
      }
#pragma unroll
      for (int r = 0; r < 16; r++) sm.x[(o + r) * LA + o + c] = xc[r];
    }
    __syncthreads();
    inverse_offdiag(sm.a, sm.x, sm.y, warp, lane);
    // T1 = T diag(beta Gamma), T2 = T diag(beta) (lower triangular, f16)
    for (int e = threadIdx.x; e < CH * CH; e += 256) {
      const int i = e >> 6, j = e & 63;
      const float t = j <= i ? sm.x[i * LA + j] : 0.0f;
      const float bj = sm.beta[j];
      sm.t1[i * L64 + j] = __float2half_rn(t * bj * __expf(sm.G[j]));
      sm.t2[i * L64 + j] = __float2half_rn(t * bj);
    }
    __syncthreads();

    // 4. W = T1 K^ (64 x 128, to shared memory) and U = T2 V (64 x DVS, in registers)
    float uacc[NT][4];
    {
      const int nw = (warp >> 2) * 64;
      float wacc[8][4];
#pragma unroll
      for (int i = 0; i < 8; i++) wacc[i][0] = wacc[i][1] = wacc[i][2] = wacc[i][3] = 0.0f;
#pragma unroll
      for (int i = 0; i < NT; i++) uacc[i][0] = uacc[i][1] = uacc[i][2] = uacc[i][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < CH / 16; ks++) {
        uint32_t at1[4], at2[4];
        ldsm_x4(a_addr(sm.t1, L64, mt * 16, ks * 16, lane), at1);
        ldsm_x4(a_addr(sm.t2, L64, mt * 16, ks * 16, lane), at2);
#pragma unroll
        for (int j2 = 0; j2 < 4; j2++) {
          uint32_t bk[4];
          ldsm_x4_t(bt_addr(sm.k, LQK, ks * 16, nw + j2 * 16, lane), bk);
          mma16816(wacc[2 * j2], at1, bk[0], bk[1]);
          mma16816(wacc[2 * j2 + 1], at1, bk[2], bk[3]);
        }
#pragma unroll
        for (int j2 = 0; j2 < NT / 2; j2++) {
          uint32_t bv[4];
          ldsm_x4_t(bt_addr(sm.v, LV, ks * 16, nbase + j2 * 16, lane), bv);
          mma16816(uacc[2 * j2], at2, bv[0], bv[1]);
          mma16816(uacc[2 * j2 + 1], at2, bv[2], bv[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 8; nt++) {
        const int row = mt * 16 + g8, col = nw + nt * 8 + 2 * tq;
        *reinterpret_cast<__half2*>(&sm.w[row * LQK + col]) = __floats2half2_rn(wacc[nt][0], wacc[nt][1]);
        *reinterpret_cast<__half2*>(&sm.w[(row + 8) * LQK + col]) = __floats2half2_rn(wacc[nt][2], wacc[nt][3]);
      }
    }
    __syncthreads();

    // 5. delta = U - W S0 and Gamma Q^ S0
    float oacc[NT][4];
    {
      float wsacc[NT][4];
#pragma unroll
      for (int i = 0; i < NT; i++)
#pragma unroll
        for (int r = 0; r < 4; r++) wsacc[i][r] = oacc[i][r] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < DK / 16; ks++) {
        uint32_t aw[4], aq[4];
        ldsm_x4(a_addr(sm.w, LQK, mt * 16, ks * 16, lane), aw);
        ldsm_x4(a_addr(sm.q, LQK, mt * 16, ks * 16, lane), aq);
#pragma unroll
        for (int j2 = 0; j2 < NT / 2; j2++) {
          uint32_t bs[4];
          ldsm_x4_t(bt_addr(sm.s, LV, ks * 16, nbase + j2 * 16, lane), bs);
          mma16816(wsacc[2 * j2], aw, bs[0], bs[1]);
          mma16816(wsacc[2 * j2 + 1], aw, bs[2], bs[3]);
          mma16816(oacc[2 * j2], aq, bs[0], bs[1]);
          mma16816(oacc[2 * j2 + 1], aq, bs[2], bs[3]);
        }
      }
      const float glast = sm.G[CH - 1];
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          const int i = mt * 16 + g8 + hf * 8, col = nbase + nt * 8 + 2 * tq;
          const float d0 = uacc[nt][2 * hf] - wsacc[nt][2 * hf], d1 = uacc[nt][2 * hf + 1] - wsacc[nt][2 * hf + 1];
          const float gi = __expf(sm.G[i]), sc = __expf(glast - sm.G[i]);
          *reinterpret_cast<__half2*>(&sm.d[i * LV + col]) = __floats2half2_rn(d0, d1);
          *reinterpret_cast<__half2*>(&sm.ds[i * LV + col]) = __floats2half2_rn(d0 * sc, d1 * sc);
          oacc[nt][2 * hf] *= gi;
          oacc[nt][2 * hf + 1] *= gi;
        }
    }
    __syncthreads();

    // 6. O = Gamma Q^ S0 + P delta, stored for the valid tokens
    {
#pragma unroll
      for (int ks = 0; ks < CH / 16; ks++) {
        uint32_t ap[4];
        ldsm_x4(a_addr(sm.p, L64, mt * 16, ks * 16, lane), ap);
#pragma unroll
        for (int j2 = 0; j2 < NT / 2; j2++) {
          uint32_t bd[4];
          ldsm_x4_t(bt_addr(sm.d, LV, ks * 16, nbase + j2 * 16, lane), bd);
          mma16816(oacc[2 * j2], ap, bd[0], bd[1]);
          mma16816(oacc[2 * j2 + 1], ap, bd[2], bd[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          const int i = mt * 16 + g8 + hf * 8, col = nbase + nt * 8 + 2 * tq;
          if (i < n)
            *reinterpret_cast<float2*>(og + (long long)(t0 + i) * H * DK + col) =
                make_float2(oacc[nt][2 * hf], oacc[nt][2 * hf + 1]);
        }
    }

    // 7. S = Gamma_C S0 + K^T (decayed delta)
    {
      const float gc = __expf(sm.G[CH - 1]);
#pragma unroll
      for (int nt = 0; nt < DVS / 8; nt++)
#pragma unroll
        for (int r = 0; r < 4; r++) sacc[nt][r] *= gc;
#pragma unroll
      for (int ks = 0; ks < CH / 16; ks++) {
        uint32_t akt[4];
        ldsm_x4_t(at_addr(sm.k, LQK, ks * 16, warp * 16, lane), akt);
#pragma unroll
        for (int j2 = 0; j2 < DVS / 16; j2++) {
          uint32_t bd[4];
          ldsm_x4_t(bt_addr(sm.ds, LV, ks * 16, j2 * 16, lane), bd);
          mma16816(sacc[2 * j2], akt, bd[0], bd[1]);
          mma16816(sacc[2 * j2 + 1], akt, bd[2], bd[3]);
        }
      }
    }
    __syncthreads();  // every warp is done reading the old f16 state and this chunk's tiles
    write_state_f16();
    __syncthreads();
  }
  // final state (f32)
  if (sout) {
#pragma unroll
    for (int nt = 0; nt < DVS / 8; nt++)
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const int row = warp * 16 + g8 + (r >> 1) * 8, col = nt * 8 + 2 * tq + (r & 1);
        sout[row * DK + col] = sacc[nt][r];
      }
  }
}

// ---------------------------------------------------------------------------------------------
// Two-phase form for a few long sequences (the engine's case: one sequence, 16 heads). Phase 1
// computes, for every (chunk, head) in parallel, everything that does not depend on the state; phase
// 2 walks the chunks of each (head, value slice) in order with only the state-dependent products.
// Per chunk and head, phase 1 writes (ChunkRec): K^ and Gamma Q^ (f16 64x128), W (f16 64x128),
// U (f32 64x128), P (f16 64x64), exp(G_C - G_i) (f32 64) and Gamma_C.
// ---------------------------------------------------------------------------------------------
struct ChunkRec {
  __half k[CH * DK];
  __half qg[CH * DK];
  __half w[CH * DK];
  float u[CH * DK];
  __half p[CH * CH];
  float dsc[CH];
  float gc;
  float pad[3];
};
static_assert(sizeof(ChunkRec) % 16 == 0, "records are copied in 16-byte pieces");

struct PrepSmem {
  __half q[CH * LQK];
  __half k[CH * LQK];
  __half v[CH * LQK];
  __half t1[CH * L64];
  __half t2[CH * L64];
  float a[CH * LA];
  float x[CH * LA];
  float y[3 * 16 * 17];
  float beta[CH], g[CH], G[CH];
};

// Phase 1: grid (chunks, heads). Inputs f16 rows as in the chunked kernel: one sequence of l tokens,
// or (chunk_tab non-null) packed sequences whose chunk c starts at token chunk_tab[2c] and holds
// chunk_tab[2c + 1] tokens. Record (c, h) is rec[h * chunks + c].
__global__ void __launch_bounds__(256, 2) gdn_prep_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                                                          int qk_stride, const __half* __restrict__ v, int v_stride,
                                                          const float* __restrict__ beta, const float* __restrict__ gl, int l,
                                                          int H, const int* __restrict__ chunk_tab, ChunkRec* __restrict__ rec) {
  extern __shared__ __align__(16) uint8_t prep_smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(prep_smem_raw);
  const int c = blockIdx.x, h = blockIdx.y;
  const int t0 = chunk_tab ? chunk_tab[2 * c] : c * CH, n = chunk_tab ? chunk_tab[2 * c + 1] : min(CH, l - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g8 = lane >> 2, tq = lane & 3;
  const int mt = warp & 3;
  ChunkRec& R = rec[(size_t)h * gridDim.x + c];
  const float qscale = rsqrtf((float)DK);

  // 1. q^, k^ (normalised), v: each warp loads its 8 rows at once, then reduces
  {
    uint2 qr[8], kr[8], vr[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int r = warp + 8 * i;
      qr[i] = kr[i] = vr[i] = make_uint2(0, 0);
      if (r < n) {
        qr[i] = *reinterpret_cast<const uint2*>(q + (long long)(t0 + r) * qk_stride + h * DK + lane * 4);
        kr[i] = *reinterpret_cast<const uint2*>(k + (long long)(t0 + r) * qk_stride + h * DK + lane * 4);
        vr[i] = *reinterpret_cast<const uint2*>(v + (long long)(t0 + r) * v_stride + h * DK + lane * 4);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int r = warp + 8 * i;
      const float4 qv = load4<__half>(reinterpret_cast<const __half*>(&qr[i]));
      const float4 kv = load4<__half>(reinterpret_cast<const __half*>(&kr[i]));
      const float sq = warp_sum(qv.x * qv.x + qv.y * qv.y + qv.z * qv.z + qv.w * qv.w);
      const float sk = warp_sum(kv.x * kv.x + kv.y * kv.y + kv.z * kv.z + kv.w * kv.w);
      const float rq = rsqrtf(sq + 1e-6f) * qscale, rk = rsqrtf(sk + 1e-6f);
      __half2* qd = reinterpret_cast<__half2*>(&sm.q[r * LQK + lane * 4]);
      __half2* kd = reinterpret_cast<__half2*>(&sm.k[r * LQK + lane * 4]);
      qd[0] = __floats2half2_rn(qv.x * rq, qv.y * rq);
      qd[1] = __floats2half2_rn(qv.z * rq, qv.w * rq);
      kd[0] = __floats2half2_rn(kv.x * rk, kv.y * rk);
      kd[1] = __floats2half2_rn(kv.z * rk, kv.w * rk);
      *reinterpret_cast<uint2*>(&sm.v[r * LQK + lane * 4]) = vr[i];
    }
  }
  if (threadIdx.x < CH) {
    const int r = threadIdx.x;
    sm.beta[r] = r < n ? beta[(long long)(t0 + r) * H + h] : 0.0f;
    sm.g[r] = r < n ? gl[(long long)(t0 + r) * H + h] : 0.0f;
  }
  __syncthreads();
  if (warp == 0) {
    const float x0 = sm.g[2 * lane], x1 = sm.g[2 * lane + 1];
    float s = x0 + x1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += u;
    }
    const float before = s - (x0 + x1);
    sm.G[2 * lane] = before + x0;
    sm.G[2 * lane + 1] = s;
  }
  __syncthreads();
  // K^ and Gamma Q^ to the record
  for (int e = threadIdx.x; e < CH * DK / 8; e += 256) {
    const int r = e >> 4, c8 = (e & 15) * 8;
    *reinterpret_cast<uint4*>(&R.k[r * DK + c8]) = *reinterpret_cast<const uint4*>(&sm.k[r * LQK + c8]);
    const __half2 gi = __float2half2_rn(__expf(sm.G[r]));
    uint4 qv = *reinterpret_cast<const uint4*>(&sm.q[r * LQK + c8]);
    __half2* q2 = reinterpret_cast<__half2*>(&qv);
#pragma unroll
    for (int j = 0; j < 4; j++) q2[j] = __hmul2(q2[j], gi);
    *reinterpret_cast<uint4*>(&R.qg[r * DK + c8]) = qv;
  }
  if (threadIdx.x < CH) {
    R.dsc[threadIdx.x] = __expf(sm.G[CH - 1] - sm.G[threadIdx.x]);
    sm.g[threadIdx.x] = sm.beta[threadIdx.x] * __expf(sm.G[threadIdx.x]);  // beta_j Gamma_j, for T1 (read after a barrier)
  }
  if (threadIdx.x == 0) R.gc = __expf(sm.G[CH - 1]);

  // 2. A and P
  {
    const int nb = (warp >> 2) * 32;
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) kk[i][j] = qk[i][j] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < DK / 16; ks++) {
      uint32_t ak[4], aq[4];
      ldsm_x4(a_addr(sm.k, LQK, mt * 16, ks * 16, lane), ak);
      ldsm_x4(a_addr(sm.q, LQK, mt * 16, ks * 16, lane), aq);
#pragma unroll
      for (int j2 = 0; j2 < 2; j2++) {
        uint32_t bk[4];
        ldsm_x4(bn_addr(sm.k, LQK, nb + j2 * 16, ks * 16, lane), bk);
        mma16816(kk[2 * j2], ak, bk[0], bk[1]);
        mma16816(kk[2 * j2 + 1], ak, bk[2], bk[3]);
        mma16816(qk[2 * j2], aq, bk[0], bk[1]);
        mma16816(qk[2 * j2 + 1], aq, bk[2], bk[3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; nt++)
#pragma unroll
      for (int hf = 0; hf < 2; hf++) {  // elements (i, j) and (i, j + 1)
        const int i = mt * 16 + g8 + hf * 8, j = nb + nt * 8 + 2 * tq;
        const float e0 = j <= i ? __expf(sm.G[i] - sm.G[j]) : 0.0f, e1 = j + 1 <= i ? __expf(sm.G[i] - sm.G[j + 1]) : 0.0f;
        sm.a[i * LA + j] = j < i ? sm.beta[i] * e0 * kk[nt][2 * hf] : 0.0f;
        sm.a[i * LA + j + 1] = j + 1 < i ? sm.beta[i] * e1 * kk[nt][2 * hf + 1] : 0.0f;
        *reinterpret_cast<__half2*>(&R.p[i * CH + j]) = __floats2half2_rn(e0 * qk[nt][2 * hf], e1 * qk[nt][2 * hf + 1]);
      }
  }
  __syncthreads();
  // 3. T = (I + A)^-1 (blocked by 16)
  if (warp < 4 && lane < 16) {
    const int o = warp * 16, cc = lane;
    float xc[16];
#pragma unroll
    for (int r = 0; r < 16; r++) {
      float v0 = r == cc ? 1.0f : 0.0f, v1 = 0.0f;
#pragma unroll
      for (int j = 0; j < r; j++)
        if (j >= cc) {
          if (j & 1) v1 -= sm.a[(o + r) * LA + o + j] * xc[j];
          else v0 -= sm.a[(o + r) * LA + o + j] * xc[j];
        }
      xc[r] = r >= cc ? v0 + v1 : 0.0f;
    }
#pragma unroll
    for (int r = 0; r < 16; r++) sm.x[(o + r) * LA + o + cc] = xc[r];
  }
  __syncthreads();
  inverse_offdiag(sm.a, sm.x, sm.y, warp, lane);
  for (int e = threadIdx.x; e < CH * CH; e += 256) {
    const int i = e >> 6, j = e & 63;
    const float t = j <= i ? sm.x[i * LA + j] : 0.0f;
    sm.t1[i * L64 + j] = __float2half_rn(t * sm.g[j]);  // beta_j Gamma_j
    sm.t2[i * L64 + j] = __float2half_rn(t * sm.beta[j]);
  }
  __syncthreads();
  // 4. W = T1 K^ (f16) and U = T2 V (f32), 64 x 128 each
  {
    const int nw = (warp >> 2) * 64;
    float wacc[8][4], uacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
      for (int r = 0; r < 4; r++) wacc[i][r] = uacc[i][r] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < CH / 16; ks++) {
      uint32_t at1[4], at2[4];
      ldsm_x4(a_addr(sm.t1, L64, mt * 16, ks * 16, lane), at1);
      ldsm_x4(a_addr(sm.t2, L64, mt * 16, ks * 16, lane), at2);
#pragma unroll
      for (int j2 = 0; j2 < 4; j2++) {
        uint32_t bk[4], bv[4];
        ldsm_x4_t(bt_addr(sm.k, LQK, ks * 16, nw + j2 * 16, lane), bk);
        ldsm_x4_t(bt_addr(sm.v, LQK, ks * 16, nw + j2 * 16, lane), bv);
        mma16816(wacc[2 * j2], at1, bk[0], bk[1]);
        mma16816(wacc[2 * j2 + 1], at1, bk[2], bk[3]);
        mma16816(uacc[2 * j2], at2, bv[0], bv[1]);
        mma16816(uacc[2 * j2 + 1], at2, bv[2], bv[3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; nt++)
#pragma unroll
      for (int hf = 0; hf < 2; hf++) {
        const int row = mt * 16 + g8 + hf * 8, col = nw + nt * 8 + 2 * tq;
        *reinterpret_cast<__half2*>(&R.w[row * DK + col]) = __floats2half2_rn(wacc[nt][2 * hf], wacc[nt][2 * hf + 1]);
        *reinterpret_cast<float2*>(&R.u[row * DK + col]) = make_float2(uacc[nt][2 * hf], uacc[nt][2 * hf + 1]);
      }
  }
}

template <int DVS>
struct ScanSmem {
  static constexpr int LV = DVS + 8;
  // double-buffered chunk records (the slice of U only)
  __half k[2][CH * LQK];
  __half qg[2][CH * LQK];
  __half w[2][CH * LQK];
  __half p[2][CH * L64];
  float u[2][CH * DVS];
  float dsc[2][CH];
  float gc[2][4];
  __half s[DK * LV];
  __half d[CH * LV];
  __half ds[CH * LV];
};

// Packed sequences of the two-phase scan: sequence b is tokens seq_off[b] .. + seq_len[b], its chunks
// are records chunk0[b] .. of every head; it starts from s_in[b] (null: zeros) and its final state
// goes to s_out[b] (null table or entry: not stored). CTA row y takes sequence order[y] (longest first).
struct ScanPacked {
  const int *seq_off = nullptr, *seq_len = nullptr, *chunk0 = nullptr, *order = nullptr;
  const float* const* s_in = nullptr;
  float* const* s_out = nullptr;
  int total_chunks = 0;
};

// Phase 2: grid (heads x 128/DVS, sequences). Walks the chunks in order; the next chunk's record is
// prefetched. One sequence: `state` in (with load_state) and out; packed: `ps`.
template <int DVS>
__global__ void __launch_bounds__(256, 1) gdn_scan_kernel(const ChunkRec* __restrict__ rec, int nchunks_one, int l, int H,
                                                          float* __restrict__ state, int load_state, float* __restrict__ o,
                                                          const ScanPacked ps) {
  constexpr int LV = ScanSmem<DVS>::LV;
  constexpr int NT = DVS / 16;
  extern __shared__ __align__(16) uint8_t scan_smem_raw[];
  ScanSmem<DVS>& sm = *reinterpret_cast<ScanSmem<DVS>*>(scan_smem_raw);
  const int NS = DK / DVS;
  const int h = blockIdx.x / NS, c0 = (blockIdx.x % NS) * DVS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g8 = lane >> 2, tq = lane & 3;
  const int mt = warp & 3, nbase = (warp >> 2) * (DVS / 2);
  const long long hoff = (long long)h * DK * DK + c0;
  const float* sin;
  float* sout;
  const ChunkRec* rh;
  int nchunks;
  long long tb = 0;  // first token of the sequence
  if (ps.seq_off) {
    const int b = ps.order[blockIdx.y];
    tb = ps.seq_off[b];
    l = ps.seq_len[b];
    nchunks = (l + CH - 1) / CH;
    rh = rec + (size_t)h * ps.total_chunks + ps.chunk0[b];
    sin = ps.s_in && ps.s_in[b] ? ps.s_in[b] + hoff : nullptr;
    sout = ps.s_out && ps.s_out[b] ? ps.s_out[b] + hoff : nullptr;
  } else {
    nchunks = nchunks_one;
    rh = rec + (size_t)h * nchunks;
    sin = load_state ? state + hoff : nullptr;
    sout = state + hoff;
  }
  float* og = o + tb * H * DK + h * DK + c0;

  auto prefetch = [&](int c, int b) {
    const ChunkRec& R = rh[c];
    for (int e = threadIdx.x; e < CH * DK / 8; e += 256) {
      const int r = e >> 4, c8 = (e & 15) * 8;
      cp_async(&sm.k[b][r * LQK + c8], &R.k[r * DK + c8], 16, 16);
      cp_async(&sm.qg[b][r * LQK + c8], &R.qg[r * DK + c8], 16, 16);
      cp_async(&sm.w[b][r * LQK + c8], &R.w[r * DK + c8], 16, 16);
    }
    for (int e = threadIdx.x; e < CH * CH / 8; e += 256) {
      const int r = e >> 3, c8 = (e & 7) * 8;
      cp_async(&sm.p[b][r * L64 + c8], &R.p[r * CH + c8], 16, 16);
    }
    for (int e = threadIdx.x; e < CH * DVS / 4; e += 256) {
      const int r = e / (DVS / 4), c4 = (e % (DVS / 4)) * 4;
      cp_async(&sm.u[b][r * DVS + c4], &R.u[r * DK + c0 + c4], 16, 16);
    }
    if (threadIdx.x < CH / 4) cp_async(&sm.dsc[b][threadIdx.x * 4], &R.dsc[threadIdx.x * 4], 16, 16);
    if (threadIdx.x == CH / 4) cp_async(&sm.gc[b][0], &R.gc, 16, 16);
    cp_async_commit();
  };

  float sacc[DVS / 8][4];
#pragma unroll
  for (int nt = 0; nt < DVS / 8; nt++)
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int row = warp * 16 + g8 + (r >> 1) * 8, col = nt * 8 + 2 * tq + (r & 1);
      sacc[nt][r] = sin ? sin[row * DK + col] : 0.0f;
    }
  auto write_state_f16 = [&]() {
#pragma unroll
    for (int nt = 0; nt < DVS / 8; nt++) {
      const int row = warp * 16 + g8, col = nt * 8 + 2 * tq;
      *reinterpret_cast<__half2*>(&sm.s[row * LV + col]) = __floats2half2_rn(sacc[nt][0], sacc[nt][1]);
      *reinterpret_cast<__half2*>(&sm.s[(row + 8) * LV + col]) = __floats2half2_rn(sacc[nt][2], sacc[nt][3]);
    }
  };
  write_state_f16();
  prefetch(0, 0);
  for (int c = 0; c < nchunks; c++) {
    const int b = c & 1;
    const int t0 = c * CH, n = min(CH, l - t0);
    cp_async_wait_all();
    __syncthreads();  // chunk c's record landed; the other buffer is free
    if (c + 1 < nchunks) prefetch(c + 1, b ^ 1);
    // delta = U - W S, O = (Gamma Q^) S
    float dacc[NT][4], oacc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++)
#pragma unroll
      for (int r = 0; r < 4; r++) dacc[i][r] = oacc[i][r] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < DK / 16; ks++) {
      uint32_t aw[4], aq[4];
      ldsm_x4(a_addr(sm.w[b], LQK, mt * 16, ks * 16, lane), aw);
      ldsm_x4(a_addr(sm.qg[b], LQK, mt * 16, ks * 16, lane), aq);
#pragma unroll
      for (int j2 = 0; j2 < NT / 2; j2++) {
        uint32_t bs[4];
        ldsm_x4_t(bt_addr(sm.s, LV, ks * 16, nbase + j2 * 16, lane), bs);
        mma16816(dacc[2 * j2], aw, bs[0], bs[1]);
        mma16816(dacc[2 * j2 + 1], aw, bs[2], bs[3]);
        mma16816(oacc[2 * j2], aq, bs[0], bs[1]);
        mma16816(oacc[2 * j2 + 1], aq, bs[2], bs[3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int hf = 0; hf < 2; hf++) {
        const int i = mt * 16 + g8 + hf * 8, col = nbase + nt * 8 + 2 * tq;
        const float2 u = *reinterpret_cast<const float2*>(&sm.u[b][i * DVS + col]);
        const float d0 = u.x - dacc[nt][2 * hf], d1 = u.y - dacc[nt][2 * hf + 1];
        const float sc = sm.dsc[b][i];
        *reinterpret_cast<__half2*>(&sm.d[i * LV + col]) = __floats2half2_rn(d0, d1);
        *reinterpret_cast<__half2*>(&sm.ds[i * LV + col]) = __floats2half2_rn(d0 * sc, d1 * sc);
      }
    __syncthreads();
    // O += P delta
#pragma unroll
    for (int ks = 0; ks < CH / 16; ks++) {
      uint32_t ap[4];
      ldsm_x4(a_addr(sm.p[b], L64, mt * 16, ks * 16, lane), ap);
#pragma unroll
      for (int j2 = 0; j2 < NT / 2; j2++) {
        uint32_t bd[4];
        ldsm_x4_t(bt_addr(sm.d, LV, ks * 16, nbase + j2 * 16, lane), bd);
        mma16816(oacc[2 * j2], ap, bd[0], bd[1]);
        mma16816(oacc[2 * j2 + 1], ap, bd[2], bd[3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int hf = 0; hf < 2; hf++) {
        const int i = mt * 16 + g8 + hf * 8, col = nbase + nt * 8 + 2 * tq;
        if (i < n)
          *reinterpret_cast<float2*>(og + (long long)(t0 + i) * H * DK + col) = make_float2(oacc[nt][2 * hf], oacc[nt][2 * hf + 1]);
      }
    // S = Gamma_C S + K^T (decayed delta)
    const float gc = sm.gc[b][0];
#pragma unroll
    for (int nt = 0; nt < DVS / 8; nt++)
#pragma unroll
      for (int r = 0; r < 4; r++) sacc[nt][r] *= gc;
#pragma unroll
    for (int ks = 0; ks < CH / 16; ks++) {
      uint32_t akt[4];
      ldsm_x4_t(at_addr(sm.k[b], LQK, ks * 16, warp * 16, lane), akt);
#pragma unroll
      for (int j2 = 0; j2 < DVS / 16; j2++) {
        uint32_t bd[4];
        ldsm_x4_t(bt_addr(sm.ds, LV, ks * 16, j2 * 16, lane), bd);
        mma16816(sacc[2 * j2], akt, bd[0], bd[1]);
        mma16816(sacc[2 * j2 + 1], akt, bd[2], bd[3]);
      }
    }
    __syncthreads();  // done with the old f16 state, delta and this chunk's buffers
    write_state_f16();
  }
  if (sout)
#pragma unroll
    for (int nt = 0; nt < DVS / 8; nt++)
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const int row = warp * 16 + g8 + (r >> 1) * 8, col = nt * 8 + 2 * tq + (r & 1);
        sout[row * DK + col] = sacc[nt][r];
      }
}

// The fixed scratch array of sd_gdn_noalloc (the two-phase scan's per-chunk records, for callers that
// cannot allocate). It belongs to this file's module: under CUDA's lazy module loading the module, and
// with it these 24 MiB, is loaded on a device the first time anything in it is used there, which the
// engine does at creation (preload_gdn) and a bare caller at its first sd_gdn / sd_gdn_noalloc call.
constexpr size_t kNoAllocScratchBytes = (size_t)24 << 20;
static __device__ __align__(256) unsigned char g_gdn_noalloc_scratch[kNoAllocScratchBytes];

// The array's device address on the current device. Host code cannot use the symbol itself (on the
// host it names a stand-in, not device memory), so the address is looked up once per device, with
// that device current, and cached.
static cudaError_t noalloc_scratch(void** out) {
  static void* addr[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gdn_noalloc_scratch);
    if (e != cudaSuccess) return e;
    addr[dev] = p;
  }
  *out = addr[dev];
  return cudaSuccess;
}

// Sets the dynamic shared-memory size of every gated-delta kernel on the current device, once per
// device. Host threads that drive different streams may reach a device's first launch together, so
// the flag is taken under a lock.
static cudaError_t set_gdn_attrs() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(gdn_chunk_kernel<32, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(GdnSmem<32>))) != cudaSuccess ||
      (e = cudaFuncSetAttribute(gdn_chunk_kernel<64, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(GdnSmem<64>))) != cudaSuccess ||
      (e = cudaFuncSetAttribute(gdn_chunk_kernel<32, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(GdnSmem<32>))) != cudaSuccess ||
      (e = cudaFuncSetAttribute(gdn_chunk_kernel<64, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(GdnSmem<64>))) != cudaSuccess ||
      (e = cudaFuncSetAttribute(gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PrepSmem))) !=
          cudaSuccess ||
      (e = cudaFuncSetAttribute(gdn_scan_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(ScanSmem<32>))) != cudaSuccess ||
      (e = cudaFuncSetAttribute(gdn_scan_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(ScanSmem<64>))) != cudaSuccess)
    return e;
  return cudaSuccess;
}
static cudaError_t ensure_gdn_attrs() {
  static bool done[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> g(mu);
  if (done[dev]) return cudaSuccess;
  if ((e = set_gdn_attrs()) == cudaSuccess) done[dev] = true;
  return e;
}

size_t gdn_two_phase_scratch(int l, int h) { return (size_t)(((long long)l + CH - 1) / CH) * h * sizeof(ChunkRec); }

// One sequence, f16 q/k/v rows: phase 1 over all (chunk, head), then the scan over (head, slice).
cudaError_t launch_gdn_two_phase(const __half* q, const __half* k, int qk_stride, const __half* v, int v_stride,
                                 const float* beta, const float* g, float* state, bool load_state, float* o, int l, int h,
                                 void* scratch, size_t scratch_bytes, cudaStream_t st) {
  if (l <= 0 || h <= 0 || scratch_bytes < gdn_two_phase_scratch(l, h)) return cudaErrorInvalidValue;
  constexpr int DVS = 32;
  cudaError_t e = ensure_gdn_attrs();
  if (e != cudaSuccess) return e;
  const int nchunks = (int)(((long long)l + CH - 1) / CH);
  ChunkRec* rec = reinterpret_cast<ChunkRec*>(scratch);
  gdn_prep_kernel<<<dim3(nchunks, h), 256, sizeof(PrepSmem), st>>>(q, k, qk_stride, v, v_stride, beta, g, l, h, nullptr, rec);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  gdn_scan_kernel<DVS><<<h * (DK / DVS), 256, sizeof(ScanSmem<DVS>), st>>>(rec, nchunks, l, h, state, load_state ? 1 : 0, o,
                                                                          ScanPacked{});
  return cudaGetLastError();
}

size_t gdn_two_phase_packed_scratch(int chunks, int h) { return (size_t)chunks * h * sizeof(ChunkRec); }

// Packed sequences, f16 q/k/v rows (token-major, sequence b at tokens seq_off[b] .. + seq_len[b]):
// phase 1 over every (chunk, head) of every sequence, then the scan over (head, slice, sequence).
// Device arrays: chunk_tab [chunks][2] (first token, tokens) of every chunk, sequences' chunks
// consecutive from chunk0[b]; order: the sequences longest first; s_in / s_out as ScanPacked.
cudaError_t launch_gdn_two_phase_packed(const __half* q, const __half* k, int qk_stride, const __half* v, int v_stride,
                                        const float* beta, const float* g, const float* const* s_in, float* const* s_out,
                                        float* o, const int* seq_off, const int* seq_len, const int* chunk0, const int* order,
                                        const int* chunk_tab, int nseq, int chunks, int h, void* scratch, size_t scratch_bytes,
                                        int num_sms, cudaStream_t st) {
  if (nseq <= 0 || chunks <= 0 || h <= 0 || scratch_bytes < gdn_two_phase_packed_scratch(chunks, h) || nseq > 65535)
    return cudaErrorInvalidValue;
  ChunkRec* rec = reinterpret_cast<ChunkRec*>(scratch);
  gdn_prep_kernel<<<dim3(chunks, h), 256, sizeof(PrepSmem), st>>>(q, k, qk_stride, v, v_stride, beta, g, 0, h, chunk_tab, rec);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  ScanPacked ps;
  ps.seq_off = seq_off, ps.seq_len = seq_len, ps.chunk0 = chunk0, ps.order = order, ps.s_in = s_in, ps.s_out = s_out;
  ps.total_chunks = chunks;
  // value slices of 64 columns once two CTAs per head and sequence fill the SMs (half the CTAs
  // re-reading each chunk's record), else of 32 (more CTAs for a few sequences)
  if ((long long)nseq * h * 2 >= num_sms)
    gdn_scan_kernel<64><<<dim3(h * 2, nseq), 256, sizeof(ScanSmem<64>), st>>>(rec, 0, 0, h, nullptr, 0, o, ps);
  else
    gdn_scan_kernel<32><<<dim3(h * 4, nseq), 256, sizeof(ScanSmem<32>), st>>>(rec, 0, 0, h, nullptr, 0, o, ps);
  return cudaGetLastError();
}

template <int DVS, typename TIn>
static cudaError_t launch_chunk(const GdnArgs<TIn>& a, int batch, cudaStream_t st) {
  auto kern = gdn_chunk_kernel<DVS, TIn>;
  const int smem = (int)sizeof(GdnSmem<DVS>);
  cudaError_t e = ensure_gdn_attrs();
  if (e != cudaSuccess) return e;
  dim3 grid(a.h * (DK / DVS), batch);
  kern<<<grid, 256, smem, st>>>(a);
  return cudaGetLastError();
}

// The chunked scan over `batch` sequences. DVS (value columns per CTA) trades redundant intra-chunk
// work for parallelism: 32 for a single sequence (64 CTAs for 16 heads), 64 for batches.
cudaError_t launch_gdn_chunked(const void* q, const void* k, int qk_stride, const void* v, int v_stride, long long seq_qk,
                               long long seq_v, bool in_f16, const float* beta, const float* g, float* state, bool load_state,
                               float* o, int l, int h, int batch, cudaStream_t st) {
  if (l <= 0 || h <= 0 || batch <= 0) return cudaErrorInvalidValue;
  const bool wide = (long long)batch * h >= 128;
  if (in_f16) {
    GdnArgs<__half> a{(const __half*)q, (const __half*)k, (const __half*)v, qk_stride, v_stride, seq_qk, seq_v,
                      beta, g, state, o, load_state ? 1 : 0, l, h};
    return wide ? launch_chunk<64>(a, batch, st) : launch_chunk<32>(a, batch, st);
  }
  GdnArgs<float> a{(const float*)q, (const float*)k, (const float*)v, qk_stride, v_stride, seq_qk, seq_v,
                   beta, g, state, o, load_state ? 1 : 0, l, h};
  return wide ? launch_chunk<64>(a, batch, st) : launch_chunk<32>(a, batch, st);
}

// Loads the gated-delta kernels on the current device (see preload_gemm), and with them this file's
// module, so the fixed scratch of sd_gdn_noalloc is committed and its address known from engine
// creation on, not at a first call made after the process has reserved its memory.
cudaError_t preload_gdn() {
  cudaError_t e = ensure_gdn_attrs();
  void* scratch = nullptr;
  if (e == cudaSuccess) e = noalloc_scratch(&scratch);
  return e;
}

// The chunked scan over `nseq` packed sequences of different lengths (sequence b: tokens seq_off[b] ..
// + seq_len[b], device arrays), sequence b starting from states[b] (a device array of pointers, the
// same one for every continuation of one prefix; a null entry: zeros), which is read and not written;
// the final state of sequence b goes to states_out[b] (null table or entry: not stored). Continuations
// of snapshots, as a batched fork runs them (one CTA walks all chunks of its sequence: for short ones).
cudaError_t launch_gdn_chunked_packed(const __half* q, const __half* k, int qk_stride, const __half* v, int v_stride,
                                      const float* beta, const float* g, const float* const* states, float* const* states_out,
                                      float* o, const int* seq_off, const int* seq_len, int nseq, int h, cudaStream_t st) {
  if (nseq <= 0 || h <= 0 || !states || nseq > 65535) return cudaErrorInvalidValue;
  GdnArgs<__half> a{q, k, v, qk_stride, v_stride, 0, 0, beta, g, nullptr, o, 1, 0, h};
  a.seq_off = seq_off;
  a.seq_len = seq_len;
  a.states = states;
  a.states_out = states_out;
  a.store_state = 0;
  return (long long)nseq * h >= 128 ? launch_chunk<64>(a, nseq, st) : launch_chunk<32>(a, nseq, st);
}

}  // namespace sd

// ---------------------------------------------------------------------------------------------
// The two-phase scan without allocation. Its per-chunk records live in the fixed device array above
// (g_gdn_noalloc_scratch): a device holds these 24 MiB from the moment this file's module loads there
// (engine creation, or the first gated-delta call) until the process exits, and every call on a
// device uses the same array.
// ---------------------------------------------------------------------------------------------
namespace sd {
namespace {
constexpr int kNoAllocRecords = (int)(kNoAllocScratchBytes / sizeof(ChunkRec));
}  // namespace
}  // namespace sd

extern "C" int32_t sd_gdn_noalloc_max_tokens(int32_t h) {
  if (h <= 0 || h > sd::kNoAllocRecords) return 0;
  return (sd::kNoAllocRecords / h) * 64;
}

extern "C" int sd_gdn_noalloc(const void* q, const void* k, int32_t qk_stride, const void* v, int32_t v_stride,
                              const void* beta, const void* g, void* state, int32_t load_state, void* o, int32_t l,
                              int32_t h, void* stream) {
  if (!q || !k || !v || !beta || !g || !state || !o || l <= 0 || h <= 0 || qk_stride % 4 || (size_t)q % 8 ||
      (size_t)k % 8) {
    sd::set_last_error("sd_gdn_noalloc: bad arguments");
    return SD_ERR_INVALID;
  }
  const long long chunks = ((long long)l + 63) / 64, records = chunks * h;
  if (records > sd::kNoAllocRecords) {
    sd::set_last_error("sd_gdn_noalloc: " + std::to_string(h) + " heads x " + std::to_string(chunks) +
                       " chunks of 64 tokens need " + std::to_string(records) + " chunk records; the fixed scratch holds " +
                       std::to_string(sd::kNoAllocRecords) + " (at most " + std::to_string(sd_gdn_noalloc_max_tokens(h)) +
                       " tokens for " + std::to_string(h) + " heads)");
    return SD_ERR_INVALID;
  }
  void* scratch = nullptr;
  cudaError_t e = sd::noalloc_scratch(&scratch);
  if (e == cudaSuccess)
    e = sd::launch_gdn_two_phase((const __half*)q, (const __half*)k, qk_stride, (const __half*)v, v_stride,
                                 (const float*)beta, (const float*)g, (float*)state, load_state != 0, (float*)o, l, h, scratch,
                                 sd::kNoAllocScratchBytes, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    sd::set_last_error(std::string("sd_gdn_noalloc: ") + cudaGetErrorString(e));
    return SD_ERR_CUDA;
  }
  return SD_OK;
}
