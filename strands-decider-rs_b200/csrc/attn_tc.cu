// Causal GQA prefill attention on the 5th-generation tensor cores (the reference's `attn`,
// src/kernels.rs:453-541, for query blocks of 128): out[t][h] = f16( softmax_j<=pos(t) (q_t . k_j / 16)
// V / (1 + exp(-gate)) ), f32 scores and accumulation, probabilities rounded to f16 as the P operand
// of the PV product, as attn.cu computes them.
//
// One CTA per (128 queries, q head); six warps:
//   warp 0     TMA: the Q tile once (128 x 256 f16, four 64-column boxes), then per block of 64 keys
//              its K tile and its V tile (64 x 256 each) into two-deep rings of their own;
//   warp 1     one thread issues tcgen05.mma: S_j = Q K_j^T (M 128, N 64, K 256: 16 MMAs, both
//              operands K-major from shared memory) into one of two S buffers in TMEM, then
//              O += P_{j-1} V_{j-1} (M 128, N 256, K 64: 4 MMAs, P from TMEM, V MN-major from shared
//              memory), so the softmax of block j overlaps the PV product of block j-1;
//   warps 2-5  softmax, one thread per query row (its TMEM lane): S row out of TMEM, causal mask,
//              row max, probabilities, row sum in registers, no shuffles; P (f16) into one of two P
//              buffers in TMEM. At the end: O out of TMEM, / row sum, sigmoid gate, f16 rows out.
// Tensor memory (512 columns): S 2 x 64, P 2 x 32, O 256.
//
// The running max is updated lazily: probabilities are taken against the max used so far, m_used,
// and O (in TMEM) is rescaled only when a row's max grows past m_used + 8 (then P <= e^8, well inside
// f16), so after the first blocks the softmax rarely touches O. The normalised result is the same;
// only the point where probabilities are rounded to f16 moves (relative rounding is unchanged).
//
// Keys of a block past the queries' reach are masked; K/V rows past the valid range read zeros (the
// tensor maps end there), so a masked key never brings a non-finite value into the PV product.
#include "common.cuh"
#include "sd_internal.h"

namespace sd {

namespace {
constexpr int TQ = 128, TK = 64, HD = 256;
constexpr int kQBox = TQ * 64 * 2;    // 16 KB: 128 rows x 64 columns
constexpr int kKVBox = TK * 64 * 2;   // 8 KB: 64 rows x 64 columns
constexpr int kQBytes = 4 * kQBox;    // 64 KB
constexpr int kKVBytes = 4 * kKVBox;  // 32 KB
constexpr int kOffK = kQBytes, kOffV = kOffK + 2 * kKVBytes, kOffBar = kOffV + 2 * kKVBytes;
// barriers
enum {
  BQ_FULL = 0,
  BK_FULL = 1,    // [2] K tile landed (TMA bytes)
  BK_EMPTY = 3,   // [2] S MMAs that read it completed
  BV_FULL = 5,    // [2]
  BV_EMPTY = 7,   // [2] PV MMAs that read it completed
  BS_FULL = 9,    // [2] S_j in TMEM
  BS_EMPTY = 11,  // [2] the softmax warps read S_j (4 arrivals)
  BP_FULL = 13,   // [2] P_j in TMEM and O rescaled (4 arrivals)
  BPV_DONE = 15,  // [2] PV_j completed (P buffer free, O updated)
  BO_FULL = 17,   // every PV completed
  BMMA_END = 18,  // every MMA issued completed (teardown)
  kBars = 19
};
constexpr int kSmem = kOffBar + kBars * 8 + 16 + 1024;
constexpr uint32_t kColS = 0, kColP = 128, kColO = 256, kTmemCols = 512;
constexpr float kLazy = 8.0f;  // rescale O once a row max grows past the one in use by this much

__device__ int g_attn_tc_err;  // error slot of calls without one

SD_DEV bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  return mbar_wait(bar, parity, abort, err ? err : &g_attn_tc_err, code);
}
SD_DEV bool wait_bar_warp(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  return mbar_wait_warp(bar, parity, abort, err ? err : &g_attn_tc_err, code);
}
SD_DEV uint32_t pack_h2f(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
}  // namespace

__global__ void __launch_bounds__(192, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, kh = h / (a.hq / a.hk);

  // this CTA's queries: q0 .. q0 + nq - 1 of their sequence (positions p + q0 + i), rows tok0 + i of
  // q / gate / out; the sequence's keys are rows kbase .. of the K/V tensors
  int q0, nq, tok0, kbase, p;
  if (a.blk) {
    const int sq = a.blk[2 * blockIdx.x];
    q0 = a.blk[2 * blockIdx.x + 1];
    nq = min(TQ, a.seq_len[sq] - q0);
    tok0 = a.seq_off[sq] + q0;
    kbase = a.seq_off[sq];
    p = 0;
  } else {
    q0 = (gridDim.x - 1 - blockIdx.x) * TQ;  // longest (latest) query blocks first
    nq = min(TQ, a.l - q0);
    tok0 = q0;
    kbase = 0;
    p = a.p;
  }
  const int nkb = (p + q0 + nq + TK - 1) / TK;

  if (threadIdx.x == 0) {
    mbar_init(&bar[BQ_FULL], 1);
    for (int s = 0; s < 2; s++) {
      mbar_init(&bar[BK_FULL + s], 1);
      mbar_init(&bar[BK_EMPTY + s], 1);
      mbar_init(&bar[BV_FULL + s], 1);
      mbar_init(&bar[BV_EMPTY + s], 1);
      mbar_init(&bar[BS_FULL + s], 1);
      mbar_init(&bar[BS_EMPTY + s], 4);
      mbar_init(&bar[BP_FULL + s], 4);
      mbar_init(&bar[BPV_DONE + s], 1);
    }
    mbar_init(&bar[BO_FULL], 1);
    mbar_init(&bar[BMMA_END], 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      mbar_arrive_expect_tx(&bar[BQ_FULL], kQBytes);
      for (int c = 0; c < 4; c++) tma_load_3d(base + c * kQBox, &qmap, &bar[BQ_FULL], c * 64, tok0, h);
      int kissued = 0, vissued = 0;
      bool ok = true;
      for (int j = 0; j < nkb && ok; j++) {
        const int s = j & 1;
        if (j >= 2 && !(ok = wait_bar(&bar[BK_EMPTY + s], ((j >> 1) - 1) & 1, abort, a.err, kErrTimeoutEmpty))) break;
        mbar_arrive_expect_tx(&bar[BK_FULL + s], kKVBytes);
        for (int c = 0; c < 4; c++)
          tma_load_3d(base + kOffK + s * kKVBytes + c * kKVBox, &kmap, &bar[BK_FULL + s], c * 64, kbase + j * TK, kh);
        kissued++;
        if (j >= 2 && !(ok = wait_bar(&bar[BV_EMPTY + s], ((j >> 1) - 1) & 1, abort, a.err, kErrTimeoutEmpty))) break;
        mbar_arrive_expect_tx(&bar[BV_FULL + s], kKVBytes);
        for (int c = 0; c < 4; c++)
          tma_load_3d(base + kOffV + s * kKVBytes + c * kKVBox, &vmap, &bar[BV_FULL + s], c * 64, kbase + j * TK, kh);
        vissued++;
      }
      // no copy may land after the CTA has left: wait (bounded) for the last ones issued
      mbar_drain(&bar[BQ_FULL], 0);
      for (int j = max(0, kissued - 2); j < kissued; j++) mbar_drain(&bar[BK_FULL + (j & 1)], (j >> 1) & 1);
      for (int j = max(0, vissued - 2); j < vissued; j++) mbar_drain(&bar[BV_FULL + (j & 1)], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(TQ, TK), idPV = idesc_f16_bmn(TQ, HD);
      bool ok = wait_bar(&bar[BQ_FULL], 0, abort, a.err, kErrTimeoutFull);
      tc_fence_after();
      for (int j = 0; j <= nkb && ok; j++) {
        if (j < nkb) {  // S_j = Q K_j^T
          const int s = j & 1;
          if (!(ok = wait_bar(&bar[BK_FULL + s], (j >> 1) & 1, abort, a.err, kErrTimeoutFull))) break;
          if (j >= 2 && !(ok = wait_bar(&bar[BS_EMPTY + s], ((j >> 1) - 1) & 1, abort, a.err, kErrTimeoutEmpty))) break;
          tc_fence_after();
          const uint8_t* kt = base + kOffK + s * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < HD / 16; kk++) {  // K 16 per MMA: +32 bytes within a 64-column box
            const uint64_t qd = sw128_desc(base + (kk >> 2) * kQBox) + 2 * (kk & 3);
            const uint64_t kd = sw128_desc(kt + (kk >> 2) * kKVBox) + 2 * (kk & 3);
            tc_mma_f16(tmem + kColS + s * TK, qd, kd, idS, kk > 0);
          }
          tc_commit(&bar[BK_EMPTY + s]);
          tc_commit(&bar[BS_FULL + s]);
        }
        if (j >= 1) {  // O += P_{j-1} V_{j-1}
          const int jj = j - 1, s = jj & 1;
          if (!(ok = wait_bar(&bar[BP_FULL + s], (jj >> 1) & 1, abort, a.err, kErrTimeoutFull))) break;
          if (!(ok = wait_bar(&bar[BV_FULL + s], (jj >> 1) & 1, abort, a.err, kErrTimeoutFull))) break;
          tc_fence_after();
          const uint8_t* vt = base + kOffV + s * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < TK / 16; kk++)  // K 16 per MMA: 16 key rows of V (two 1024-byte groups)
            tc_mma_f16_ts(tmem + kColO, tmem + kColP + s * (TK / 2) + kk * 8, sw128_mn_desc(vt + kk * 2048, kKVBox), idPV,
                          (jj | kk) != 0);
          tc_commit(&bar[BV_EMPTY + s]);
          tc_commit(&bar[BPV_DONE + s]);
        }
      }
      if (ok) tc_commit(&bar[BO_FULL]);
      // every MMA issued has completed before TMEM is released
      tc_commit(&bar[BMMA_END]);
      mbar_drain(&bar[BMMA_END], 0);
    }
  } else {
    // softmax: thread = query row r (TMEM lane r; warp w may access lanes 32 (w % 4) .. + 31)
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
    const int pos = p + q0 + r;  // the last key this query sees
    float m_used = -INFINITY, lsum = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkb && ok; j++) {
      const int s = j & 1;
      if (!(ok = wait_bar_warp(&bar[BS_FULL + s], (j >> 1) & 1, abort, a.err, kErrTimeoutFull))) break;
      tc_fence_after();
      uint32_t sv[TK];
      tmem_ld32(tmem + lanes + kColS + s * TK, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
      tmem_ld32(tmem + lanes + kColS + s * TK + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[BS_EMPTY + s]);
      // scores (1/sqrt(256) = 1/16, exact), causal mask, row max
      float x[TK];
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < TK; c++) {
        const float v = __uint_as_float(sv[c]) * 0.0625f;
        x[c] = j * TK + c <= pos ? v : -INFINITY;
        mx = fmaxf(mx, x[c]);
      }
      const bool resc = mx > m_used + kLazy;  // first block: m_used = -inf
      float alpha = 1.0f;
      if (resc) {
        alpha = j == 0 ? 0.0f : __expf(m_used - mx);
        m_used = mx;
        lsum *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
        // O rescale (the warp together: TMEM loads and stores are warp-wide): after PV_{j-1}, before PV_j
        if (!(ok = wait_bar_warp(&bar[BPV_DONE + ((j - 1) & 1)], ((j - 1) >> 1) & 1, abort, a.err, kErrTimeoutAccum))) break;
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < HD; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(tmem + lanes + kColO + c0, o);
          tc_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; c++) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(tmem + lanes + kColO + c0, o);
        }
        tc_wait_st();
      }
      // probabilities against m_used, rounded to f16 for the PV product; the row sum in f32
      uint32_t pk[TK / 2];
      float ps = 0.0f;
#pragma unroll
      for (int c = 0; c < TK; c += 2) {
        const float p0 = __expf(x[c] - m_used), p1 = __expf(x[c + 1] - m_used);
        ps += p0 + p1;
        pk[c / 2] = pack_h2f(p0, p1);
      }
      lsum += ps;
      // P buffer s was read by PV_{j-2}
      if (j >= 2 && !(ok = wait_bar_warp(&bar[BPV_DONE + s], ((j >> 1) - 1) & 1, abort, a.err, kErrTimeoutAccum))) break;
      tc_fence_after();
      tmem_st32(tmem + lanes + kColP + s * (TK / 2), pk);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[BP_FULL + s]);
    }
    if (ok && wait_bar_warp(&bar[BO_FULL], 0, abort, a.err, kErrTimeoutAccum)) {
      tc_fence_after();
      const float il = 1.0f / lsum;
      const int t = tok0 + r;
#pragma unroll 1
      for (int c0 = 0; c0 < HD; c0 += 32) {
        uint32_t o[32];
        tmem_ld32(tmem + lanes + kColO + c0, o);
        tc_wait_ld();
        if (r < nq) {
          uint32_t hv[16];
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float g[8];
            if (a.gate) {
              const uint4 gr = *reinterpret_cast<const uint4*>(a.gate + (size_t)t * a.gstride + a.goff + h * a.gstep + c0 + c);
              const __half2* g2 = reinterpret_cast<const __half2*>(&gr);
#pragma unroll
              for (int i = 0; i < 4; i++) {
                const float2 f = __half22float2(g2[i]);
                g[2 * i] = f.x, g[2 * i + 1] = f.y;
              }
            }
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              float x0 = __uint_as_float(o[c + i]) * il, x1 = __uint_as_float(o[c + i + 1]) * il;
              if (a.gate) {
                x0 = x0 / (1.0f + __expf(-g[i]));
                x1 = x1 / (1.0f + __expf(-g[i + 1]));
              }
              hv[(c + i) / 2] = pack_h2f(x0, x1);
            }
          }
          uint4* dst = reinterpret_cast<uint4*>(a.out + (size_t)t * a.hq * HD + h * HD + c0);
#pragma unroll
          for (int k4 = 0; k4 < 4; k4++) dst[k4] = make_uint4(hv[4 * k4], hv[4 * k4 + 1], hv[4 * k4 + 2], hv[4 * k4 + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

cudaError_t preload_attention_tc() {
  return cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
}

// Query blocks of 128 for the tensor-core kernel; q [hq][qrows][256], k / v [hk][krows][256] with
// krows_valid rows readable per head (later rows read zeros).
cudaError_t launch_attention_tc(const __half* q, int qrows, const __half* k, const __half* v, int krows, int krows_valid,
                                const AttnTcArgs& a, int nblk, cudaStream_t st) {
  if (nblk <= 0 || nblk > 65535 || a.hq <= 0 || a.hq > 65535 || a.hk <= 0 || a.hq % a.hk || qrows <= 0 || krows_valid <= 0 ||
      krows_valid > krows || ((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16)
    return cudaErrorInvalidValue;
  if (a.gate && (a.gstride % 8 || a.goff % 8 || a.gstep % 8 || (uintptr_t)a.gate % 16)) return cudaErrorInvalidValue;
  static bool attr[kMaxDevices] = {};  // the shared-memory size, once per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = preload_attention_tc();
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  CUtensorMap qm, km, vm;
  if (make_map_3d(&qm, q, HD, qrows, a.hq, HD, (long long)qrows * HD, TQ) != 0 ||
      make_map_3d(&km, k, HD, krows_valid, a.hk, HD, (long long)krows * HD, TK) != 0 ||
      make_map_3d(&vm, v, HD, krows_valid, a.hk, HD, (long long)krows * HD, TK) != 0)
    return cudaErrorInvalidValue;
  attn_tc_kernel<<<dim3(nblk, a.hq), 192, kSmem, st>>>(qm, km, vm, a);
  return cudaGetLastError();
}

}  // namespace sd
