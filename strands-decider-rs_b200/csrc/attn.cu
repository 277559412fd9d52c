// Causal GQA attention with the sigmoid output gate (the reference's `attn`, src/kernels.rs:453-541):
// out[t][h] = f16( softmax_j<=p+t (q_t . k_j / sqrt(HD)) V / (1 + exp(-gate)) ), with q pre-scaled by
// 1/sqrt(HD) and rounded to f16 as the reference stages it (src/kernels.rs:475-476), f32 scores and
// accumulation, probabilities rounded to f16 as the P operand of the PV product.
//
// Flash-style: one CTA per (64 queries, q head), 4 warps of 16 query rows; keys in blocks of 32 with
// an online softmax in registers. Q, K and V tiles are staged in padded shared memory (row stride
// 264 halves, so ldmatrix rows fall in distinct banks); K/V blocks are double-buffered with cp.async
// and rows past the last valid key are zero-filled. When the (query block, head) grid is too small to
// fill the GPU (a short continuation over a long prefix) the keys are split across CTAs as well: each
// split writes its unnormalised output with its row max and sum (f32), and attn_combine merges the
// splits (rescaled to the largest max) and applies the gate. In packed mode (AttnPacked) the queries are
// several sequences packed back to back, each continuing one cached prefix: the keys of a sequence are
// the prefix's (from the cache) and then its own (from tail buffers), never another sequence's.
#include <algorithm>

#include <atomic>

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
                    int lt, int hq, int hk, float* __restrict__ part_o, float* __restrict__ part_ml, const AttnPacked pk) {
  extern __shared__ __align__(16) uint8_t smem[];
  __half* sq = reinterpret_cast<__half*>(smem);
  __half* skv = reinterpret_cast<__half*>(smem + kSmemQ);  // [2][K | V]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, kh = h / (hq / hk);
  // t0: first query of the block within its sequence; tok0: its row in q, gate, out (and the tails)
  int t0, nq, tok0;
  if (pk.blk) {
    const int sq = pk.blk[2 * blockIdx.x];
    t0 = pk.blk[2 * blockIdx.x + 1];
    nq = min(BQ, pk.seq_len[sq] - t0);
    tok0 = pk.seq_off[sq] + t0;
    if (pk.kp) {  // this sequence's own prefix: its length and its K/V rows
      p = pk.plen[sq];
      lt = p;
      k = pk.kp[sq];
      v = pk.vp[sq];
    }
  } else {
    t0 = (gridDim.x - 1 - blockIdx.x) * BQ;  // longest (latest) query blocks first
    nq = min(BQ, l - t0);
    tok0 = t0;
  }
  const int tail0 = tok0 - t0 - p;  // tail row of key p (packed mode)
  const int kend = p + t0 + nq;     // keys [0, kend)
  const int nkb = (kend + BKV - 1) / BKV;
  // this CTA's share of the key blocks (all of them unless the keys are split: blockIdx.z of gridDim.z)
  const int per = (nkb + gridDim.z - 1) / gridDim.z;
  const int kb0 = min(nkb, (int)blockIdx.z * per), kb1 = min(nkb, kb0 + per);

  // Q tile, scaled by 1/sqrt(256) = 1/16 (exact in f16) and rounded to f16.
  for (int e = threadIdx.x; e < BQ * HD / 8; e += 128) {
    const int r = e / (HD / 8), c8 = (e % (HD / 8)) * 8;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < nq) {
      val = *reinterpret_cast<const uint4*>(q + ((size_t)h * l + tok0 + r) * HD + c8);
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
      const __half *ks = k, *vs = v;
      size_t off = ((size_t)kh * lt + (ok ? j : 0)) * HD + c8;
      if (pk.blk && j >= p) {  // this sequence's own keys (past the last one: row 0 of the tails, not read)
        ks = pk.kt, vs = pk.vt;
        off = ((size_t)kh * pk.T + (ok ? tail0 + j : 0)) * HD + c8;
      }
      cp_async16(smem_u32(dk + r * LDS + c8), ks + off, ok);
      cp_async16(smem_u32(dv + r * LDS + c8), vs + off, ok);
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

  if (kb0 < kb1) load_kv(kb0, 0);
  for (int kb = kb0; kb < kb1; kb++) {
    const int buf = (kb - kb0) & 1;
    if (kb + 1 < kb1) {
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
    // the running max; a row with no visible key yet (possible in a split that starts past it) keeps
    // -1e30, and its probabilities are taken against 0, so they are exp(-1e30) = 0, not exp(0)
    const float mn0 = fmaxf(mrow[0], mx0), mn1 = fmaxf(mrow[1], mx1);
    const float mr0 = mn0 < -1e29f ? 0.0f : mn0, mr1 = mn1 < -1e29f ? 0.0f : mn1;
    const float al0 = __expf(mrow[0] - mr0), al1 = __expf(mrow[1] - mr1);
    float sum0 = 0.0f, sum1 = 0.0f;
    uint32_t pa[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; nt++) {
      const float p0 = __expf(s[nt][0] - mr0), p1 = __expf(s[nt][1] - mr0);
      const float p2 = __expf(s[nt][2] - mr1), p3 = __expf(s[nt][3] - mr1);
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

  if (gridDim.z > 1) {
    // split keys: the unnormalised output and (max, sum) of each row, for attn_combine
#pragma unroll
    for (int half = 0; half < 2; half++) {
      const int r = row0 + half * 8;
      if (r >= nq) continue;
      const size_t row = ((size_t)blockIdx.z * hq + h) * l + tok0 + r;
#pragma unroll
      for (int nt = 0; nt < HD / 8; nt++)
        *reinterpret_cast<float2*>(part_o + row * HD + nt * 8 + 2 * tq) = make_float2(o[nt][2 * half], o[nt][2 * half + 1]);
      if (tq == 0) *reinterpret_cast<float2*>(part_ml + row * 2) = make_float2(mrow[half], lrow[half]);
    }
    return;
  }

  // out = O / l * sigmoid(gate), f16
  const float il0 = 1.0f / lrow[0], il1 = 1.0f / lrow[1];
#pragma unroll
  for (int half = 0; half < 2; half++) {
    const int r = row0 + half * 8;
    if (r >= nq) continue;
    const int t = tok0 + r;
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

// Merges the key splits of one (token, head) row per warp: out = sum_z e^(m_z - M) O_z /
// sum_z e^(m_z - M) l_z, then the sigmoid gate, f16. Lane i holds dimensions 8i .. 8i + 7.
__global__ void attn_combine(const float* __restrict__ part_o, const float* __restrict__ part_ml, int splits, int l, int hq,
                             const __half* __restrict__ gate, int gstride, int goff, int gstep, __half* __restrict__ out) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= l * hq) return;
  const int h = row / l, t = row % l;
  float mmax = -1e30f;
  for (int z = 0; z < splits; z++) mmax = fmaxf(mmax, part_ml[(((size_t)z * hq + h) * l + t) * 2]);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0}, lsum = 0.0f;
  for (int z = 0; z < splits; z++) {
    const size_t r = ((size_t)z * hq + h) * l + t;
    const float2 ml = *reinterpret_cast<const float2*>(part_ml + r * 2);
    const float w = ml.y > 0.0f ? __expf(ml.x - mmax) : 0.0f;
    lsum += w * ml.y;
    const float4 a = *reinterpret_cast<const float4*>(part_o + r * HD + lane * 8);
    const float4 b = *reinterpret_cast<const float4*>(part_o + r * HD + lane * 8 + 4);
    acc[0] += w * a.x, acc[1] += w * a.y, acc[2] += w * a.z, acc[3] += w * a.w;
    acc[4] += w * b.x, acc[5] += w * b.y, acc[6] += w * b.z, acc[7] += w * b.w;
  }
  const float il = 1.0f / lsum;
  uint32_t hv[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float x0 = acc[2 * i] * il, x1 = acc[2 * i + 1] * il;
    if (gate) {
      const float2 gf = __half22float2(
          *reinterpret_cast<const __half2*>(gate + (size_t)t * gstride + goff + h * gstep + lane * 8 + 2 * i));
      x0 = x0 / (1.0f + __expf(-gf.x));
      x1 = x1 / (1.0f + __expf(-gf.y));
    }
    hv[i] = pack_h2(x0, x1);
  }
  *reinterpret_cast<uint4*>(out + (size_t)t * hq * HD + h * HD + lane * 8) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
}

// Loads the attention kernels on the current device (see preload_gemm).
cudaError_t preload_attention() {
  cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes a;
  return cudaFuncGetAttributes(&a, attn_combine);
}

size_t attention_split_bytes(int l, int hq, int splits) { return (size_t)splits * hq * l * (HD + 2) * sizeof(float); }

// Key splits for `qblocks` query blocks over at most `keys` keys: none while the (query block, head)
// grid fills the SMs, else enough to reach about two CTAs per SM, with at least four key blocks (128
// keys) per split.
static int splits_for(int qblocks, int keys, int hq, int num_sms) {
  const int ctas = qblocks * hq;
  if (ctas >= num_sms) return 1;
  const int nkb = (keys + BKV - 1) / BKV;
  return std::max(1, std::min({(2 * num_sms + ctas - 1) / ctas, nkb / 4, 32}));
}
int attention_splits(int l, int p, int hq, int num_sms) { return splits_for((l + BQ - 1) / BQ, p + l, hq, num_sms); }
int attention_splits_packed(int nblk, int p, int max_len, int hq, int num_sms) {
  return splits_for(nblk, p + max_len, hq, num_sms);
}

cudaError_t launch_attention(const __half* q, const __half* k, const __half* v, const __half* gate, int gstride, int goff,
                             int gstep, __half* out, int l, int p, int lt, int hq, int hk, int hd, int splits, float* ws,
                             size_t ws_bytes, cudaStream_t st) {
  if (hd != HD || hq % hk != 0 || l <= 0 || splits < 1) return cudaErrorInvalidValue;
  if (splits > 1 && (!ws || ws_bytes < attention_split_bytes(l, hq, splits))) return cudaErrorInvalidValue;
  static std::atomic<bool> attr[kMaxDevices] = {};  // setting it twice is harmless; the flag only saves the call
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  dim3 grid((l + BQ - 1) / BQ, hq, splits);
  float* part_o = ws;
  float* part_ml = ws ? ws + (size_t)splits * hq * l * HD : nullptr;
  attn_fwd_kernel<<<grid, 128, kSmem, st>>>(q, k, v, gate, gstride, goff, gstep, out, l, p, lt, hq, hk, part_o, part_ml,
                                            AttnPacked{});
  if (splits == 1) return cudaGetLastError();
  const int rows = l * hq;
  attn_combine<<<(rows + 3) / 4, 128, 0, st>>>(part_o, part_ml, splits, l, hq, gate, gstride, goff, gstep, out);
  return cudaGetLastError();
}

cudaError_t launch_attention_packed(const __half* q, const __half* k, const __half* v, const __half* gate, int gstride,
                                    int goff, int gstep, __half* out, int T, int p, int lt, int hq, int hk, int hd,
                                    const AttnPacked& pk, int nblk, int splits, float* ws, size_t ws_bytes, cudaStream_t st) {
  if (hd != HD || hq % hk != 0 || T <= 0 || nblk <= 0 || splits < 1 || !pk.blk) return cudaErrorInvalidValue;
  if (splits > 1 && (!ws || ws_bytes < attention_split_bytes(T, hq, splits))) return cudaErrorInvalidValue;
  static std::atomic<bool> attr[kMaxDevices] = {};  // setting it twice is harmless; the flag only saves the call
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  dim3 grid(nblk, hq, splits);
  float* part_o = ws;
  float* part_ml = ws ? ws + (size_t)splits * hq * T * HD : nullptr;
  attn_fwd_kernel<<<grid, 128, kSmem, st>>>(q, k, v, gate, gstride, goff, gstep, out, T, p, lt, hq, hk, part_o, part_ml, pk);
  if (splits == 1) return cudaGetLastError();
  const int rows = T * hq;
  attn_combine<<<(rows + 3) / 4, 128, 0, st>>>(part_o, part_ml, splits, T, hq, gate, gstride, goff, gstep, out);
  return cudaGetLastError();
}

}  // namespace sd
