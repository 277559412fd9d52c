// Causal GQA prefill attention on the 5th-generation tensor cores (the reference's `attn`,
// src/kernels.rs:453-541, for query blocks of 128): out[t][h] = f16( softmax_j<=pos(t) (q_t . k_j / 16)
// V / (1 + exp(-gate)) ), f32 scores and accumulation, probabilities rounded to f16 as the P operand
// of the PV product, as attn.cu computes them.
//
// One CTA per (128 queries, q head), keys in blocks of 128; six warps:
//   warp 0     TMA: the Q tile (128 x 256 f16, four 64-column boxes) once, then the K and V tiles of
//              every key block into one ring of nine 16 KB slots, in the order the MMAs read them
//              (K_0, K_1, V_0, K_2, V_1, ...): a K tile as four boxes of 128 keys x 64 columns, a V
//              tile as four chunks of 32 keys x 256 columns, so a slot frees as soon as the MMAs of
//              its part are done and the next tiles stream in behind them;
//   warp 1     one thread issues tcgen05.mma: S_j = Q K_j^T (M 128, N 128, K 256: 16 MMAs, both
//              operands K-major from shared memory) into one of two S buffers in TMEM, then
//              O += P_{j-1} V_{j-1} (M 128, N 256, K 128: 8 MMAs, P from TMEM, V MN-major from shared
//              memory), so the softmax of block j overlaps the PV product of block j-1;
//   warps 2-5  softmax, one thread per query row (its TMEM lane): the S row out of TMEM, causal mask,
//              row max, probabilities and row sum in registers, no shuffles; P (f16) written over
//              the first half of the same S buffer. At the end: O out of TMEM, / row sum, sigmoid
//              gate, f16 rows out.
// Tensor memory (512 columns): S/P 2 x 128, O 256. An S buffer is rewritten (S_{j+2}) only after the
// PV product that read its P (PV_j) has completed.
//
// The running max is updated lazily: probabilities are taken against the max used so far, m_used,
// and O (in TMEM) is rescaled only when a row's max grows past m_used + 8 (then P <= e^8, well inside
// f16), so after the first blocks the softmax rarely touches O. The normalised result is the same;
// only the point where probabilities are rounded to f16 moves (relative rounding is unchanged).
//
// Keys of a block past the queries' reach are masked; K/V rows past the valid range read zeros (the
// tensor maps end there), so a masked key never brings a non-finite value into the PV product.
#include <atomic>

#include "common.cuh"
#include "sd_internal.h"

namespace sd {

namespace {
constexpr int TQ = 128, TK = 128, HD = 256;
constexpr int kQBox = TQ * 64 * 2;  // 16 KB: 128 rows x 64 columns
constexpr int kQBytes = 4 * kQBox;  // 64 KB
constexpr int kSlot = 16384;        // one ring slot: a K box (128 keys x 64) or a V chunk (32 keys x 256)
constexpr int kVSub = 4096;         // a V chunk's 64-column part (32 keys x 64)
constexpr int kSlots = 9;
constexpr int kOffRing = kQBytes, kOffBar = kOffRing + kSlots * kSlot;
// barriers
enum {
  BQ_FULL = 0,
  B_FULL = 1,                // [kSlots] a slot's tile part landed (TMA bytes)
  B_EMPTY = 1 + kSlots,      // [kSlots] the MMAs that read it completed
  BS_FULL = 1 + 2 * kSlots,  // [2] S_j in TMEM
  BP_FULL = BS_FULL + 2,     // [2] P_j in TMEM and O rescaled (4 arrivals)
  BPV_DONE = BP_FULL + 2,    // [2] PV_j completed (its S buffer free, O updated)
  BO_FULL = BPV_DONE + 2,    // every PV completed
  BMMA_END = BO_FULL + 1,    // every MMA issued completed (teardown)
  kBars = BMMA_END + 1
};
constexpr int kSmem = kOffBar + kBars * 8 + 16 + 1024;
constexpr uint32_t kColO = 256, kTmemCols = 512;  // S/P buffers at columns 0 and 128
// Scores are handled in the log2 domain: y = s / 16 * log2(e), probabilities 2^(y - m).
constexpr float kScaleL2 = 0.0625f * 1.4426950408889634f;
constexpr float kLazy = 8.0f * 1.4426950408889634f;  // rescale O once a row max grows past the one in use by e^8
constexpr int kThreads = 192;

__device__ int g_attn_tc_err;  // error slot of calls without one

SD_DEV bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  return mbar_wait<false>(bar, parity, abort, err ? err : &g_attn_tc_err, code);
}
SD_DEV bool wait_bar_warp(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  return mbar_wait_warp<false>(bar, parity, abort, err ? err : &g_attn_tc_err, code);
}
SD_DEV float ex2(float x) {  // 2^x (the hardware's approximate exponential, as __expf uses)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
SD_DEV uint32_t pack_h2f(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const AttnTcArgs a) {
  grid_dep_wait();  // launched as a programmatic dependent (launch_dependent): inputs ready from here
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base + kOffRing;
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Blocks are dispatched in linear order (x fastest). The query-block index is made the slowest
  // varying one, so the longest query blocks of every head and batch element start first and the
  // short ones fill the tail (the x order alone would run all of one head's blocks before the next
  // head's longest).
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int hb = gridDim.y * gridDim.z, bx = lin / hb;
  const int h = (lin % hb) % gridDim.y, kh = h / (a.hq / a.hk);
  const int bz = (lin % hb) / gridDim.y;  // batch element (single-sequence mode): q / k / v slabs bz * heads + head

  // this CTA's queries: q0 .. q0 + nq - 1 of their sequence (positions p + q0 + i), rows tok0 + i of
  // q / gate / out; the sequence's keys are rows kbase .. of the K/V tensors
  int q0, nq, tok0, kbase, p;
  if (a.blk) {
    const int sq = a.blk[2 * bx];
    q0 = a.blk[2 * bx + 1];
    nq = min(TQ, a.seq_len[sq] - q0);
    tok0 = a.seq_off[sq] + q0;
    kbase = a.kbase_tab ? a.kbase_tab[sq] : a.seq_off[sq];
    p = a.plen ? a.plen[sq] : 0;
  } else {
    q0 = (gridDim.x - 1 - bx) * TQ;  // longest (latest) query blocks first
    nq = min(TQ, a.l - q0);
    tok0 = q0;
    kbase = 0;
    p = a.p;
  }
  const int nkb = (p + q0 + nq + TK - 1) / TK;

  if (threadIdx.x == 0) {
    mbar_init(&bar[BQ_FULL], 1);
    for (int s = 0; s < kSlots; s++) {
      mbar_init(&bar[B_FULL + s], 1);
      mbar_init(&bar[B_EMPTY + s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&bar[BS_FULL + b], 1);
      mbar_init(&bar[BP_FULL + b], 4);
      mbar_init(&bar[BPV_DONE + b], 1);
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
      for (int c = 0; c < 4; c++) tma_load_3d(base + c * kQBox, &qmap, &bar[BQ_FULL], c * 64, tok0, bz * a.hq + h);
      // ring items in MMA order: K_0, then per block j >= 1 K_j and V_{j-1}, then V_{nkb-1}
      int it = 0;
      bool ok = true;
      auto slot_wait = [&]() -> int {  // the next slot, once its previous tile part is consumed
        const int s = it % kSlots, u = it / kSlots;
        if (u >= 1 && !wait_bar(&bar[B_EMPTY + s], (u - 1) & 1, abort, a.err, kErrTimeoutEmpty)) return -1;
        return s;
      };
      for (int j = 0; j <= nkb && ok; j++) {
        if (j < nkb)
          for (int c = 0; c < 4 && ok; c++, it++) {  // K_j box c: keys j*128 .., columns 64c ..
            const int s = slot_wait();
            if (s < 0) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bar[B_FULL + s], kSlot);
            tma_load_3d(ring + s * kSlot, &kmap, &bar[B_FULL + s], c * 64, kbase + j * TK, bz * a.hk + kh);
          }
        if (j >= 1)
          for (int c = 0; c < 4 && ok; c++, it++) {  // V_{j-1} chunk c: keys (j-1)*128 + 32c .., all columns
            const int s = slot_wait();
            if (s < 0) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bar[B_FULL + s], kSlot);
            for (int hb = 0; hb < 4; hb++)
              tma_load_3d(ring + s * kSlot + hb * kVSub, &vmap, &bar[B_FULL + s], hb * 64, kbase + (j - 1) * TK + c * 32,
                          bz * a.hk + kh);
          }
      }
      // no copy may land after the CTA has left: wait (bounded) for the last ones issued
      mbar_drain(&bar[BQ_FULL], 0);
      for (int i = max(0, it - kSlots); i < it; i++) mbar_drain(&bar[B_FULL + i % kSlots], (i / kSlots) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(TQ, TK), idPV = idesc_f16_bmn(TQ, HD);
      // descriptors of the first box of each tile; a box, a k step or a slot is an add to the start
      // address field (16-byte units)
      const uint64_t qd0 = sw128_desc(base), rd0 = sw128_desc(ring), vd0 = sw128_mn_desc(ring, kVSub);
      bool ok = wait_bar(&bar[BQ_FULL], 0, abort, a.err, kErrTimeoutFull);
      tc_fence_after();
      int it = 0;
      for (int j = 0; j <= nkb && ok; j++) {
        if (j < nkb) {  // S_j = Q K_j^T into buffer j & 1, once PV_{j-2} (which read its P) is done
          const int b = j & 1;
          if (j >= 2 && !(ok = wait_bar(&bar[BPV_DONE + b], ((j >> 1) - 1) & 1, abort, a.err, kErrTimeoutEmpty))) break;
          for (int c = 0; c < 4; c++, it++) {
            const int s = it % kSlots;
            if (!(ok = wait_bar(&bar[B_FULL + s], (it / kSlots) & 1, abort, a.err, kErrTimeoutFull))) break;
            tc_fence_after();
            const uint64_t kd = rd0 + (uint64_t)(s * (kSlot >> 4));
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++)  // K 16 per MMA: +32 bytes within the 64-column box
              tc_mma_f16(tmem + b * TK, qd0 + (uint64_t)(c * (kQBox >> 4) + 2 * k4), kd + (uint64_t)(2 * k4), idS,
                         (c | k4) != 0);
            tc_commit(&bar[B_EMPTY + s]);
          }
          if (!ok) break;
          tc_commit(&bar[BS_FULL + b]);
        }
        if (j >= 1) {  // O += P_{j-1} V_{j-1}
          const int jj = j - 1, b = jj & 1;
          if (!(ok = wait_bar(&bar[BP_FULL + b], (jj >> 1) & 1, abort, a.err, kErrTimeoutFull))) break;
          for (int c = 0; c < 4; c++, it++) {
            const int s = it % kSlots;
            if (!(ok = wait_bar(&bar[B_FULL + s], (it / kSlots) & 1, abort, a.err, kErrTimeoutFull))) break;
            tc_fence_after();
            const uint64_t vd = vd0 + (uint64_t)(s * (kSlot >> 4));
#pragma unroll
            for (int k2 = 0; k2 < 2; k2++)  // K 16 per MMA: 8 TMEM columns of P, 16 key rows of V (2048 bytes)
              tc_mma_f16_ts(tmem + kColO, tmem + b * TK + (c * 2 + k2) * 8, vd + (uint64_t)(k2 * (2048 >> 4)), idPV,
                            (jj | c | k2) != 0);
            tc_commit(&bar[B_EMPTY + s]);
          }
          if (!ok) break;
          tc_commit(&bar[BPV_DONE + b]);
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
      const int b = j & 1;
      const uint32_t sb = tmem + lanes + b * TK;
      if (!(ok = wait_bar_warp(&bar[BS_FULL + b], (j >> 1) & 1, abort, a.err, kErrTimeoutFull))) break;
      tc_fence_after();
      uint32_t sv[TK];
#pragma unroll
      for (int c = 0; c < TK; c += 32) tmem_ld32(sb + c, *reinterpret_cast<uint32_t(*)[32]>(&sv[c]));
      tc_wait_ld();
      // causal mask (only where the block reaches past a row of this warp), row max of the raw
      // scores; in the log2 domain y = s * kScaleL2 (1/16 = 1/sqrt(256) and log2(e))
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (j * TK + TK - 1 <= p + q0 + (warp & 3) * 32) {  // every key of the block is visible to the warp
#pragma unroll
        for (int c = 0; c < TK; c++) m4[c & 3] = fmaxf(m4[c & 3], __uint_as_float(sv[c]));
      } else {
#pragma unroll
        for (int c = 0; c < TK; c++) {
          if (j * TK + c > pos) sv[c] = __float_as_uint(-INFINITY);
          m4[c & 3] = fmaxf(m4[c & 3], __uint_as_float(sv[c]));
        }
      }
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * kScaleL2;
      const bool resc = mx > m_used + kLazy;  // first block: m_used = -inf
      float alpha = 1.0f;
      if (resc) {
        alpha = j == 0 ? 0.0f : ex2(m_used - mx);
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
      // probabilities 2^(y - m_used), rounded to f16 for the PV product (packed in place over the
      // scores already read); the row sum in f32
      float ps4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < TK; c += 2) {
        const float p0 = ex2(fmaf(__uint_as_float(sv[c]), kScaleL2, -m_used));
        const float p1 = ex2(fmaf(__uint_as_float(sv[c + 1]), kScaleL2, -m_used));
        ps4[(c >> 1) & 3] += p0 + p1;
        sv[c / 2] = pack_h2f(p0, p1);
      }
      lsum += (ps4[0] + ps4[1]) + (ps4[2] + ps4[3]);
      // P over the first 64 columns of this S buffer (its scores are all in registers now)
      tmem_st32(sb, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
      tmem_st32(sb + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[BP_FULL + b]);
    }
    // this row's gate, all of it at once (one memory latency, overlapping the last PV product; the
    // registers of the scores are free now)
    const size_t t = (size_t)bz * a.l + tok0 + r;  // row of gate / out
    uint4 grow[HD / 8];
    if (a.gate && r < nq) {
      const uint4* gsrc = reinterpret_cast<const uint4*>(a.gate + t * a.gstride + a.goff + h * a.gstep);
#pragma unroll
      for (int i = 0; i < HD / 8; i++) grow[i] = gsrc[i];
    }
    // out = O / row sum x sigmoid(gate), f16, each thread its own row (staging the tile in shared
    // memory for row-contiguous stores measured 8% slower)
    const bool done = ok && wait_bar_warp(&bar[BO_FULL], 0, abort, a.err, kErrTimeoutAccum);
    if (done) {
      tc_fence_after();
      const float il = 1.0f / lsum;
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 32) {
        uint32_t o[32];
        tmem_ld32(tmem + lanes + kColO + c0, o);
        tc_wait_ld();
        {
          uint32_t hv[16];
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            float g[8];
            if (a.gate) {
              const __half2* g2 = reinterpret_cast<const __half2*>(&grow[(c0 + c) / 8]);
#pragma unroll
              for (int i = 0; i < 4; i++) {
                const float2 f = __half22float2(g2[i]);
                g[2 * i] = f.x, g[2 * i + 1] = f.y;
              }
            }
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              float x0 = __uint_as_float(o[c + i]) * il, x1 = __uint_as_float(o[c + i + 1]) * il;
              if (a.gate) {  // x sigmoid(gate) (fast division: within 2 ulp, far below the f16 rounding that follows)
                x0 = __fdividef(x0, 1.0f + __expf(-g[i]));
                x1 = __fdividef(x1, 1.0f + __expf(-g[i + 1]));
              }
              hv[(c + i) / 2] = pack_h2f(x0, x1);
            }
          }
          if (r < nq) {
            uint4* dst = reinterpret_cast<uint4*>(a.out + t * a.hq * HD + h * HD + c0);
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++) dst[k4] = make_uint4(hv[4 * k4], hv[4 * k4 + 1], hv[4 * k4 + 2], hv[4 * k4 + 3]);
          }
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

// Query blocks of 128 for the tensor-core kernel; q [batch][hq][qrows][256], k / v [batch][hk][krows][256]
// with krows_valid rows readable per head (later rows read zeros); gate / out rows batch-major.
cudaError_t launch_attention_tc(const __half* q, int qrows, const __half* k, const __half* v, int krows, int krows_valid,
                                const AttnTcArgs& a, int nblk, cudaStream_t st) {
  if (nblk <= 0 || nblk > 65535 || a.hq <= 0 || a.hq > 65535 || a.hk <= 0 || a.hq % a.hk || qrows <= 0 || krows_valid <= 0 ||
      krows_valid > krows || ((uintptr_t)q | (uintptr_t)k | (uintptr_t)v) % 16 || a.batch < 1 || a.batch > 65535 ||
      (a.blk && a.batch != 1))
    return cudaErrorInvalidValue;
  if (a.gate && (a.gstride % 8 || a.goff % 8 || a.gstep % 8 || (uintptr_t)a.gate % 16)) return cudaErrorInvalidValue;
  static std::atomic<bool> attr[kMaxDevices] = {};  // the shared-memory size, once per device (setting it twice is harmless)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = preload_attention_tc();
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  CUtensorMap qm, km, vm;
  if (make_map_3d(&qm, q, HD, qrows, a.batch * a.hq, HD, (long long)qrows * HD, TQ) != 0 ||
      make_map_3d(&km, k, HD, krows_valid, a.batch * a.hk, HD, (long long)krows * HD, TK) != 0 ||
      make_map_3d(&vm, v, HD, krows_valid, a.batch * a.hk, HD, (long long)krows * HD, 32) != 0)
    return cudaErrorInvalidValue;
  return launch_dependent(attn_tc_kernel, dim3(nblk, a.hq, a.batch), dim3(kThreads), kSmem, st, qm, km, vm, a);
}

cudaError_t take_attn_tc_err(int* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_attn_tc_err, sizeof(int));
  const int zero = 0;
  if (e == cudaSuccess && *code != 0) e = cudaMemcpyToSymbol(g_attn_tc_err, &zero, sizeof(int));
  return e;
}

}  // namespace sd
