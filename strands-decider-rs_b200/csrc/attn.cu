// Causal GQA attention with the sigmoid output gate (the reference's `attn`, src/kernels.rs:453-541):
// out[t][h] = f16( softmax_j<=p+t (q_t . k_j / sqrt(HD)) V / (1 + exp(-gate)) ), with q pre-scaled by
// 1/sqrt(HD) and rounded to f16 as the reference stages it (src/kernels.rs:475-476), f32 scores and
// accumulation, probabilities rounded to f16 as the P operand of the PV product.
//
// Flash-style: one CTA per (64 queries, q head), 4 warps of 16 query rows; keys in blocks of 32 with
// an online softmax in registers. Q, K and V tiles are staged in padded shared memory (row stride
// 264 halves, so ldmatrix rows fall in distinct banks); K/V blocks are double-buffered with cp.async
// and rows past the last valid key are zero-filled.
#include "common.cuh"
#include "sd_internal.h"

namespace sd {

namespace {
constexpr int HD = 256;
constexpr int BQ = 64;
constexpr int BKV = 32;
constexpr int LDS = HD + 8;  // padded row stride in halves
constexpr int kSmemQ = BQ * LDS * 2;
constexpr int kSmemKV = BKV * LDS * 2;
constexpr int kSmem = kSmemQ + 4 * kSmemKV;  // Q + 2 x (K, V)

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0 source bytes: the 16 destination bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
}  // namespace

__global__ void __launch_bounds__(128, 2)
    attn_fwd_kernel(const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                    const __half* __restrict__ gate, int gstride, int goff, int gstep, __half* __restrict__ out, int l, int p,
                    int lt, int hq, int hk) {
  extern __shared__ __align__(16) uint8_t smem[];
  __half* sq = reinterpret_cast<__half*>(smem);
  __half* skv = reinterpret_cast<__half*>(smem + kSmemQ);  // [2][K | V]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest (latest) query blocks first
  const int h = blockIdx.y, kh = h / (hq / hk);
  const int t0 = qb * BQ;
  const int nq = min(BQ, l - t0);
  const int kend = p + t0 + nq;  // keys [0, kend)
  const int nkb = (kend + BKV - 1) / BKV;

  // Q tile, scaled by 1/sqrt(256) = 1/16 (exact in f16) and rounded to f16.
  for (int e = threadIdx.x; e < BQ * HD / 8; e += 128) {
    const int r = e / (HD / 8), c8 = (e % (HD / 8)) * 8;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < nq) {
      val = *reinterpret_cast<const uint4*>(q + ((size_t)h * l + t0 + r) * HD + c8);
      __half2* v2 = reinterpret_cast<__half2*>(&val);
#pragma unroll
      for (int i = 0; i < 4; i++) v2[i] = __hmul2(v2[i], __float2half2_rn(0.0625f));
    }
    *reinterpret_cast<uint4*>(sq + r * LDS + c8) = val;
  }

  auto load_kv = [&](int kb, int buf) {
    __half* dk = skv + buf * 2 * BKV * LDS;
    __half* dv = dk + BKV * LDS;
    for (int e = threadIdx.x; e < BKV * HD / 8; e += 128) {
      const int r = e / (HD / 8), c8 = (e % (HD / 8)) * 8;
      const int j = kb * BKV + r;
      const bool ok = j < kend;
      const size_t off = ((size_t)kh * lt + (ok ? j : 0)) * HD + c8;
      cp_async16(smem_u32(dk + r * LDS + c8), k + off, ok);
      cp_async16(smem_u32(dv + r * LDS + c8), v + off, ok);
    }
    cp_async_commit();
  };

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float mrow[2] = {-1e30f, -1e30f}, lrow[2] = {0.0f, 0.0f};
  const int g = lane >> 2, tq = lane & 3;
  const int row0 = warp * 16 + g;          // CTA rows of this thread: row0, row0 + 8
  const int lim0 = p + t0 + row0, lim1 = lim0 + 8;  // last key each may see

  load_kv(0, 0);
  for (int kb = 0; kb < nkb; kb++) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_kv(kb + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __half* sk = skv + buf * 2 * BKV * LDS;
    const __half* sv = sk + BKV * LDS;

    // S = Q K^T for 16 rows x 32 keys
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; kk++) {
      uint32_t a0, a1, a2, a3;
      {
        const int mat = lane >> 3;
        const int r = warp * 16 + (mat & 1) * 8 + (lane & 7);
        const int c = kk * 16 + (mat >> 1) * 8;
        ldsm_x4(smem_u32(sq + r * LDS + c), a0, a1, a2, a3);
      }
#pragma unroll
      for (int nb = 0; nb < 2; nb++) {
        uint32_t b0, b1, b2, b3;
        const int mat = lane >> 3;
        const int r = nb * 16 + (mat >> 1) * 8 + (lane & 7);
        const int c = kk * 16 + (mat & 1) * 8;
        ldsm_x4(smem_u32(sk + r * LDS + c), b0, b1, b2, b3);
        mma16816(s[2 * nb], a0, a1, a2, a3, b0, b1);
        mma16816(s[2 * nb + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // causal mask and online softmax (rows row0 and row0 + 8 of this thread)
    float mx0 = -1e30f, mx1 = -1e30f;
#pragma unroll
    for (int nt = 0; nt < 4; nt++) {
      const int j = kb * BKV + nt * 8 + 2 * tq;
      if (j > lim0) s[nt][0] = -1e30f;
      if (j + 1 > lim0) s[nt][1] = -1e30f;
      if (j > lim1) s[nt][2] = -1e30f;
      if (j + 1 > lim1) s[nt][3] = -1e30f;
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(mrow[0], mx0), mn1 = fmaxf(mrow[1], mx1);
    const float al0 = __expf(mrow[0] - mn0), al1 = __expf(mrow[1] - mn1);
    float sum0 = 0.0f, sum1 = 0.0f;
    uint32_t pa[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; nt++) {
      const float p0 = __expf(s[nt][0] - mn0), p1 = __expf(s[nt][1] - mn0);
      const float p2 = __expf(s[nt][2] - mn1), p3 = __expf(s[nt][3] - mn1);
      sum0 += p0 + p1;
      sum1 += p2 + p3;
      pa[nt][0] = pack_h2(p0, p1);
      pa[nt][1] = pack_h2(p2, p3);
    }
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);
    lrow[0] = lrow[0] * al0 + sum0;
    lrow[1] = lrow[1] * al1 + sum1;
    mrow[0] = mn0;
    mrow[1] = mn1;
#pragma unroll
    for (int i = 0; i < HD / 8; i++) {
      o[i][0] *= al0;
      o[i][1] *= al0;
      o[i][2] *= al1;
      o[i][3] *= al1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BKV / 16; kk++) {
      const uint32_t a0 = pa[2 * kk][0], a1 = pa[2 * kk][1], a2 = pa[2 * kk + 1][0], a3 = pa[2 * kk + 1][1];
#pragma unroll
      for (int nb = 0; nb < HD / 16; nb++) {
        uint32_t b0, b1, b2, b3;
        const int mat = lane >> 3;
        const int r = kk * 16 + (mat & 1) * 8 + (lane & 7);
        const int c = nb * 16 + (mat >> 1) * 8;
        ldsm_x4_t(smem_u32(sv + r * LDS + c), b0, b1, b2, b3);
        mma16816(o[2 * nb], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * nb + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }

  // out = O / l * sigmoid(gate), f16
  const float il0 = 1.0f / lrow[0], il1 = 1.0f / lrow[1];
#pragma unroll
  for (int half = 0; half < 2; half++) {
    const int r = row0 + half * 8;
    if (r >= nq) continue;
    const int t = t0 + r;
    const float il = half ? il1 : il0;
#pragma unroll
    for (int nt = 0; nt < HD / 8; nt++) {
      const int d = nt * 8 + 2 * tq;
      float x0 = o[nt][2 * half] * il, x1 = o[nt][2 * half + 1] * il;
      if (gate) {
        const __half2 gg = *reinterpret_cast<const __half2*>(gate + (size_t)t * gstride + goff + h * gstep + d);
        const float2 gf = __half22float2(gg);
        x0 = x0 / (1.0f + __expf(-gf.x));
        x1 = x1 / (1.0f + __expf(-gf.y));
      }
      *reinterpret_cast<__half2*>(out + (size_t)t * hq * HD + h * HD + d) = __floats2half2_rn(x0, x1);
    }
  }
}

cudaError_t launch_attention(const __half* q, const __half* k, const __half* v, const __half* gate, int gstride, int goff,
                             int gstep, __half* out, int l, int p, int lt, int hq, int hk, int hd, cudaStream_t st) {
  if (hd != HD || hq % hk != 0 || l <= 0) return cudaErrorInvalidValue;
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  dim3 grid((l + BQ - 1) / BQ, hq);
  attn_fwd_kernel<<<grid, 128, kSmem, st>>>(q, k, v, gate, gstride, goff, gstep, out, l, p, lt, hq, hk);
  return cudaGetLastError();
}

}  // namespace sd
