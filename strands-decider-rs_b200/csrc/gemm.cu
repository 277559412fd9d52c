// Dequantizing GEMM on the 5th-generation tensor cores: Y[m][n] = sum_k A[m][k] W[n][k], with W
// stored as the reference's int4 group-32 symmetric blocks (src/kernels.rs:545-576, `matmul_tiled`
// at src/kernels.rs:640-709 and `matmul_coop` at :716-804 are the kernels it replaces).
//
// The weights are the MMA's M side (128 rows per tile) and the tokens its N side (BN columns, up to
// 192), so one dequantized weight tile serves up to 192 tokens. The dequantized weights never touch
// shared memory: they go from registers into tensor memory, which tcgen05.mma reads its A operand
// from; only the activations (the B operand) are staged in shared memory. Persistent and
// warp-specialised:
//   raw producer  bulk-copies the packed weight k-tiles of each stage (codes + scales, 4608 bytes a
//                 k-tile, contiguous in the tile layout) into the raw ring, one copy and one barrier;
//   act producer  TMA-loads the activation k-tiles of a stage (BN x 64 f16 each, 128-byte swizzle);
//   dequantizers  NG groups of four warps, taking stages in turn: each thread reads one weight row of
//                 each k-tile of the stage from the raw ring (freeing the slot once read), dequantizes
//                 its 64 values and stores them into its TMEM lane (32 columns of f16 pairs);
//   MMA issuer    one thread: tcgen05.mma (M 128, N BN, K 16, A from TMEM, B from shared memory)
//                 into a TMEM accumulator;
//   epilogue      four warps read the accumulator out of TMEM (each its 32-lane quarter), transpose it
//                 through shared memory and store f16 token rows (or the SwiGLU of gate/up row pairs,
//                 or f32 split-K partials).
// A stage holds KS k-tiles of both operands behind one barrier (the act producer's byte count plus one
// arrival per dequantizing warp) and is released by one tcgen05.commit, so the MMA thread waits once
// and commits once per 4 KS MMAs. The raw ring runs ahead on its own barriers. TMEM holds two
// accumulators (one tile's epilogue overlaps the next tile's main loop) and the A ring.
//
// Numerics: the dequantized weight is (q - 8) * scale rounded to f16, as the reference's tiled
// kernel computes it (src/kernels.rs:671); products accumulate in f32; the output is rounded to f16.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cooperative_groups.h>

#include "common.cuh"
#include "sd_internal.h"

namespace cg = cooperative_groups;

namespace sd {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kTileCodes = kBM * kBK / 2;          // 4096 bytes of int4 codes
constexpr int kTileScales = kBM * (kBK / 32) * 2;  // 512 bytes of f16 scales
constexpr int kTileBytes = kTileCodes + kTileScales;  // a symmetric weight's k-tile
constexpr int kTileBias = kBM * (kBK / 32) * 2;        // f16 biases of an asymmetric weight's k-tile
constexpr int kTileBytesMax = kTileBytes + kTileBias;
constexpr int kHalfCodes = kTileCodes / 2;  // codes of k-group 0 of every row, then of k-group 1
constexpr int kACols = kBK / 2;             // TMEM columns of one dequantized k-tile (f16 pairs)

// WIDE: two k-tiles per stage at BN 192 (two stages, two dequantization groups; the TMEM A ring keeps
// its four k-tiles), so the MMA thread waits and commits once per 8 MMAs. Measured on B200: +3% on the
// gate_up GEMM with its SwiGLU epilogue, -2% on the down projection, so only the SwiGLU GEMM uses it.
template <int BN, int WIDE = 0>
struct GemmCfg {
  // k-tiles per stage, stages, dequantization groups (no more than stages), raw ring slots of one
  // stage's packed weights each (deeper for short prompts, whose weights stream from HBM once)
  static constexpr int KS = BN >= 192 && !WIDE ? 1 : 2;
  static constexpr int S = WIDE ? 2 : (BN >= 64 ? 4 : 6);
  static constexpr int NG = WIDE ? 2 : 4;
  static constexpr int SR = WIDE ? 8 : (BN >= 192 ? 16 : (BN >= 128 ? 8 : 12));
  static constexpr int kRawSlot = KS * kTileBytesMax;
  static constexpr int kWarps = 2 + 4 * NG + 4 + 1;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kWarpAct = 0, kWarpMma = 1, kWarpDq0 = 2, kWarpEpi0 = 2 + 4 * NG, kWarpRaw = kWarpEpi0 + 4;
  static constexpr int kAccCols = BN < 32 ? 32 : BN;  // one accumulator buffer
  static constexpr int kACol0 = 2 * kAccCols;         // the A ring follows the two accumulators
  static constexpr int kTmemUsed = kACol0 + S * KS * kACols;
  static constexpr int kTmemCols = kTmemUsed <= 256 ? 256 : 512;
  static constexpr size_t kB = (size_t)BN * kBK * 2;  // one k-tile of activations, f16
  static constexpr size_t kStage = KS * kB;
  static constexpr size_t kOffRaw = S * kStage;
  static constexpr size_t kOffStg = kOffRaw + (size_t)SR * kRawSlot;
  static constexpr int kStgBytesPerWarp = 32 * 40 * 2;  // 32 x 32 f16 (row stride 40) or 16 x 32 f32 (row stride 36)
  static constexpr size_t kOffBar = kOffStg + 4 * kStgBytesPerWarp;
  static constexpr int kBars = 2 * SR + 2 * S + 4 + 1;
  static constexpr size_t kBytes = kOffBar + kBars * 8 + 16;
  static constexpr size_t kSmem = kBytes + 1024;  // room to align the base to 1024 bytes
  static_assert(kSmem <= 232448, "shared memory per CTA");
  static_assert(kTmemUsed <= 512, "tensor memory columns");
  static_assert(kThreads <= 1024, "threads per CTA");
  static_assert(BN % 32 == 0 && BN <= 256, "the epilogue reads 32 token columns at a time");
  static_assert(S >= 2 && NG <= S, "stage ring: a group waits for the stage NG before its own");
  // A raw ring slot is reused every SR stages; the groups take stages in turn, so this keeps every use
  // of a slot with one group. Otherwise a group could poll a slot whose previous use (another group's
  // stage) has not landed yet and take that older phase, of the same parity, for its own.
  static_assert(SR % NG == 0, "raw ring: each slot belongs to one group");
};

// kEpiAdd: the f16-rounded outputs are added into the f32 rows at `ws` (ldy floats apart): the
// residual stream x += f16(A W^T), the reference's matmul-then-add_norm (src/kernels.rs:93-120) with
// the add done here.
enum Epi { kEpiStore = 0, kEpiSilu = 1, kEpiPartial = 2, kEpiAdd = 3 };
// The configuration a kernel instantiation uses.
template <int BN, int EPI>
using CfgOf = GemmCfg<BN, (EPI == kEpiSilu && BN >= 192) ? 1 : 0>;

// The SwiGLU of one output: gate and up are each rounded to f16 first, as the reference stores them.
SD_DEV float swiglu(float gate, float up) {
  const float g = __half2float(__float2half_rn(gate)), u = __half2float(__float2half_rn(up));
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

struct TileGrid {
  int ntiles, mtiles, splits, kps, KT;
  int mmajor;  // tile order: 0, weight tiles outermost; 1, token tiles outermost
  __host__ __device__ int count() const { return ntiles * mtiles * splits; }
  // Consecutive tiles share the weight tile (same n-tile, all m-tiles and splits next to each other),
  // so the CTAs running at once read a few weight tiles and every activation tile: right while the
  // activations stay in L2. With mmajor they share the token tile instead (all n-tiles of one m-tile
  // next to each other): the activations stream from HBM once while the weights stay in L2.
  __device__ void decode(int t, int& nt, int& mt, int& sp, int& kt0, int& nk) const {
    if (mmajor) {
      mt = t / (ntiles * splits);
      const int r = t % (ntiles * splits);
      nt = r / splits;
      sp = r % splits;
    } else {
      nt = t / (mtiles * splits);
      const int r = t % (mtiles * splits);
      mt = r / splits;
      sp = r % splits;
    }
    kt0 = sp * kps;
    nk = max(0, min(KT, kt0 + kps) - kt0);
  }
};

// Persistent: each CTA walks tiles blockIdx.x, +gridDim.x, ...; the rings run across tile boundaries.
// Every role walks the same sequence: tiles with work, their stages (KS k-tiles each, the last one of a
// tile possibly fewer) and k-tiles, so stage and k-tile counters agree between roles.
template <int BN, int EPI>
__global__ void __launch_bounds__(CfgOf<BN, EPI>::kThreads, 1)
    gemm_q4_tc(const __grid_constant__ CUtensorMap act_map, const uint8_t* __restrict__ wt, int M, int N, int tile_bytes,
               TileGrid tg, __half* __restrict__ y, int ldy, float* __restrict__ ws, int* err) {
  using Cfg = CfgOf<BN, EPI>;
  constexpr int KS = Cfg::KS, S = Cfg::S, SR = Cfg::SR, NG = Cfg::NG;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sraw = base + Cfg::kOffRaw;
  uint8_t* sstg = base + Cfg::kOffStg;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(base + Cfg::kOffBar);
  uint64_t* raw_empty = raw_full + SR;
  uint64_t* full = raw_empty + SR;     // [S] operands of a stage landed / written
  uint64_t* empty = full + S;          // [S] the stage's MMAs completed
  uint64_t* acc_full = empty + S;      // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* mma_done = acc_empty + 2;  // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntile_total = tg.count();

  if (threadIdx.x == 0) {
    for (int s = 0; s < SR; s++) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 4);  // the four warps of a dequantization group
    }
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 4 + 1);  // a dequantization group's warps + the act producer's byte count
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // the four epilogue warps
    }
    mbar_init(mma_done, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == Cfg::kWarpMma) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int KT = tg.KT;

  if (warp == Cfg::kWarpRaw) {
    // one thread: the packed weight k-tiles of every stage, one copy per stage into the raw ring
    if (lane == 0) {
      int si = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x) {
        int nt, mt, sp, kt0, nk;
        tg.decode(t, nt, mt, sp, kt0, nk);
        const uint8_t* wtile = wt + (size_t)nt * KT * tile_bytes;
        for (int i = 0; i < nk; i += KS, si++) {
          const int rs = si % SR, kc = min(KS, nk - i);
          if (si >= SR && !mbar_wait(&raw_empty[rs], ((si / SR) & 1) ^ 1, abort, err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)(kc * tile_bytes));
          bulk_load(sraw + rs * Cfg::kRawSlot, wtile + (size_t)(kt0 + i) * tile_bytes, kc * tile_bytes, &raw_full[rs]);
        }
      }
      for (int j = max(0, si - SR); j < si; j++) mbar_drain(&raw_full[j % SR], (j / SR) & 1);
    }
  } else if (warp == Cfg::kWarpAct) {
    // one thread: the activation k-tiles of each stage, one barrier per stage
    if (lane == 0) {
      prefetch_tmap(&act_map);
      grid_dep_wait();  // the activations are the previous kernel's output
      int si = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x) {
        int nt, mt, sp, kt0, nk;
        tg.decode(t, nt, mt, sp, kt0, nk);
        for (int i = 0; i < nk; i += KS, si++) {
          const int s = si % S, kc = min(KS, nk - i);
          if (si >= S && !mbar_wait(&empty[s], ((si / S) & 1) ^ 1, abort, err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sb = base + s * Cfg::kStage;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(kc * Cfg::kB));
          for (int j = 0; j < kc; j++) tma_load_2d(sb + j * Cfg::kB, &act_map, &full[s], (kt0 + i + j) * kBK, mt * BN);
        }
      }
      for (int j = max(0, si - S); j < si; j++) mbar_drain(&full[j % S], (j / S) & 1);
    }
  } else if (warp == Cfg::kWarpMma) {
    // one thread: one wait and one commit per stage; accumulator buffer = local tile index & 1
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kBM, BN);
      int si = 0, lt = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x) {
        int nt, mt, sp, kt0, nk;
        tg.decode(t, nt, mt, sp, kt0, nk);
        if (nk == 0) continue;
        lt++;  // tiles with work, in order
        const int buf = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, abort, err, kErrTimeoutEmpty)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * Cfg::kAccCols;
        for (int i = 0; i < nk; i += KS, si++) {
          const int s = si % S, kc = min(KS, nk - i);
          if (!mbar_wait(&full[s], (si / S) & 1, abort, err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sb = base + s * Cfg::kStage;
          const uint32_t a0 = tmem + Cfg::kACol0 + s * KS * kACols;
          for (int j = 0; j < kc; j++) {
            const uint64_t bd = sw128_desc(sb + j * Cfg::kB);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; kk++)  // K 16 per MMA: 8 TMEM columns of A, +32 bytes (+2) of B
              tc_mma_f16_ts(acc, a0 + j * kACols + kk * 8, bd + 2 * kk, idesc, (i | j | kk) != 0);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
      }
      // every MMA issued has completed before TMEM is released
      tc_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else if (warp < Cfg::kWarpEpi0) {
    // dequantization: group g takes the stages with si % NG == g; thread i of warp w owns weight row
    // (w % 4) * 32 + i, the TMEM lane this warp may write
    const int g = (warp - Cfg::kWarpDq0) >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16) + Cfg::kACol0;
    int si = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x) {
      int nt, mt, sp, kt0, nk;
      tg.decode(t, nt, mt, sp, kt0, nk);
      for (int i = 0; i < nk && ok; i += KS, si++) {
        if (si % NG != g) continue;
        const int s = si % S, rs = si % SR, kc = min(KS, nk - i);
        if (!mbar_wait_warp(&raw_full[rs], (si / SR) & 1, abort, err, kErrTimeoutFull)) {
          ok = false;
          break;
        }
        for (int j = 0; j < kc; j++) {
          const uint8_t* raw = sraw + rs * Cfg::kRawSlot + j * tile_bytes;
          const uint4 c0 = *reinterpret_cast<const uint4*>(raw + r * 16);
          const uint4 c1 = *reinterpret_cast<const uint4*>(raw + kHalfCodes + r * 16);
          const __half2 sc = *reinterpret_cast<const __half2*>(raw + kTileCodes + r * 4);
          const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          uint32_t v[32];  // column c: elements (2c, 2c + 1) of this row's 64
          if (tile_bytes == kTileBytes) {
#pragma unroll
            for (int ch = 0; ch < 8; ch++) {
              const __half2 sc2 = ch < 4 ? __low2half2(sc) : __high2half2(sc);
#pragma unroll
              for (int e = 0; e < 4; e++) v[ch * 4 + e] = h2_as_u32(dq_pair(w[ch], e, sc2));
            }
          } else {  // asymmetric: q * scale + bias
            const __half2 bi = *reinterpret_cast<const __half2*>(raw + kTileBytes + r * 4);
#pragma unroll
            for (int ch = 0; ch < 8; ch++) {
              const __half2 sc2 = ch < 4 ? __low2half2(sc) : __high2half2(sc);
              const __half2 bi2 = ch < 4 ? __low2half2(bi) : __high2half2(bi);
#pragma unroll
              for (int e = 0; e < 4; e++) v[ch * 4 + e] = h2_as_u32(dq_pair_affine(w[ch], e, sc2, bi2));
            }
          }
          if (j == kc - 1) {
            // the stage's codes are in registers (the results depend on them): refill the raw slot
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rs]);
          }
          if (j == 0 && si >= S) {
            if (!mbar_wait_warp(&empty[s], ((si / S) & 1) ^ 1, abort, err, kErrTimeoutEmpty)) {
              ok = false;
              break;
            }
            tc_fence_after();  // the MMAs that read this slot are complete
          }
          tmem_st32(lane_base + (s * KS + j) * kACols, v);
        }
        if (!ok) break;
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
    }
  } else if (warp < Cfg::kWarpRaw) {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (weight rows of the tile), transposes
    // through shared memory and stores token rows with 16-byte stores
    grid_dep_wait();  // the outputs (and x) may still be in use by the previous kernel until it completes
    const int q = warp & 3;
    uint8_t* stg = sstg + (warp - Cfg::kWarpEpi0) * Cfg::kStgBytesPerWarp;
    int lt = -1;
    for (int t = blockIdx.x; t < ntile_total; t += gridDim.x) {
      int nt, mt, sp, kt0, nk;
      tg.decode(t, nt, mt, sp, kt0, nk);
      if (nk == 0) continue;
      lt++;
      const int buf = lt & 1;
      if (!mbar_wait_warp(&acc_full[buf], (lt >> 1) & 1, abort, err, kErrTimeoutAccum)) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * Cfg::kAccCols + ((uint32_t)(q * 32) << 16);
      const int n0 = nt * kBM + q * 32;  // first weight row of this warp
      if (EPI == kEpiStore || EPI == kEpiSilu) {
        __half* st = reinterpret_cast<__half*>(stg);  // [32 tokens][40]
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          const int mbase = mt * BN + c0;
          if (mbase >= M) break;
          uint32_t v[32];
          tmem_ld32(acc + c0, v);
          tc_wait_ld();
          if (EPI == kEpiStore) {
#pragma unroll
            for (int j = 0; j < 32; j++) st[j * 40 + lane] = __float2half_rn(__uint_as_float(v[j]));
            __syncwarp();
            const int m = mbase + lane;
            if (m < M) {
              const uint4* src = reinterpret_cast<const uint4*>(st + lane * 40);
              __half* dst = y + (size_t)m * ldy + n0;
              if (n0 + 32 <= N) {
#pragma unroll
                for (int k4 = 0; k4 < 4; k4++) reinterpret_cast<uint4*>(dst)[k4] = src[k4];
              } else {
                for (int k2 = 0; k2 < 32 && n0 + k2 < N; k2++) dst[k2] = st[lane * 40 + k2];
              }
            }
          } else {
            // rows interleaved as (gate j, up j): even lanes hold gate, odd lanes up. For the token
            // pair (2p, 2p+1) the even lane computes token 2p and the odd lane token 2p+1, after one
            // exchange: the even lane sends its gate of token 2p+1, the odd lane its up of token 2p.
            const int odd = lane & 1;
#pragma unroll
            for (int p = 0; p < 16; p++) {
              const float a0 = __uint_as_float(v[2 * p]), a1 = __uint_as_float(v[2 * p + 1]);
              const float other = __shfl_xor_sync(0xffffffffu, odd ? a0 : a1, 1);
              const float g = odd ? other : a0;
              const float u = odd ? a1 : other;
              st[(2 * p + odd) * 40 + (lane >> 1)] = __float2half_rn(swiglu(g, u));
            }
            __syncwarp();
            const int m = mbase + lane;
            if (m < M && n0 < N) {
              const uint4* src = reinterpret_cast<const uint4*>(st + lane * 40);
              uint4* dst = reinterpret_cast<uint4*>(y + (size_t)m * ldy + (n0 >> 1));
              dst[0] = src[0];
              dst[1] = src[1];
            }
          }
          __syncwarp();
        }
      } else if (EPI == kEpiAdd) {
        float* st = reinterpret_cast<float*>(stg);  // [16 tokens][36], f16-rounded
        // four tokens per instruction, eight lanes a token's 32 outputs (whole 128-byte lines); the x
        // rows of the next 16 tokens are loaded while these are added, so the loads' latency overlaps
        const int ch = (lane & 7) * 4;
        auto x_at = [&](int mbase, int r4) -> float* {
          const int m = mbase + 4 * r4 + (lane >> 3);
          return m < M && n0 + ch < N ? ws + (size_t)m * ldy + n0 + ch : nullptr;  // N is a multiple of 4
        };
        float4 cur[4], nxt[4];
#pragma unroll
        for (int r4 = 0; r4 < 4; r4++)
          if (const float* p = x_at(mt * BN, r4)) cur[r4] = *reinterpret_cast<const float4*>(p);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          const int mbase = mt * BN + c0;
          if (mbase >= M) break;
          if (c0 + 16 < BN) {
#pragma unroll
            for (int r4 = 0; r4 < 4; r4++)
              if (const float* p = x_at(mbase + 16, r4)) nxt[r4] = *reinterpret_cast<const float4*>(p);
          }
          uint32_t v[16];
          tmem_ld16(acc + c0, v);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j++) st[j * 36 + lane] = __half2float(__float2half_rn(__uint_as_float(v[j])));
          __syncwarp();
#pragma unroll
          for (int r4 = 0; r4 < 4; r4++) {
            if (float* p = x_at(mbase, r4)) {
              const float4 a = *reinterpret_cast<const float4*>(st + (4 * r4 + (lane >> 3)) * 36 + ch);
              float4 xv = cur[r4];
              xv.x += a.x, xv.y += a.y, xv.z += a.z, xv.w += a.w;
              *reinterpret_cast<float4*>(p) = xv;
            }
            cur[r4] = nxt[r4];
          }
          __syncwarp();
        }
      } else {
        float* st = reinterpret_cast<float*>(stg);  // [16 tokens][36]
        float* part = ws + (size_t)sp * M * N;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          const int mbase = mt * BN + c0;
          if (mbase >= M) break;
          uint32_t v[16];
          tmem_ld16(acc + c0, v);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j++) st[j * 36 + lane] = __uint_as_float(v[j]);
          __syncwarp();
          const int m = mbase + (lane >> 1), hb = (lane & 1) * 16;
          if (m < M) {
            const float* src = st + (lane >> 1) * 36 + hb;
            float* dst = part + (size_t)m * N + n0 + hb;
            if (n0 + hb + 16 <= N) {
#pragma unroll
              for (int k4 = 0; k4 < 4; k4++) reinterpret_cast<float4*>(dst)[k4] = reinterpret_cast<const float4*>(src)[k4];
            } else {
              for (int k2 = 0; k2 < 16 && n0 + hb + k2 < N; k2++) dst[k2] = src[k2];
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == Cfg::kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// Split-K finish: sums the splits' f32 partials in split order (deterministic), then f16 (or the
// SwiGLU of interleaved gate/up rows, or f16 added into the f32 rows at xadd). Rows blockIdx.y,
// + gridDim.y, ...; each thread takes four partial columns (16-byte loads; N is a multiple of 8) and
// stores four outputs, or two with SwiGLU.
__global__ void __launch_bounds__(256) gemm_finish(const float* __restrict__ ws, int splits, int M, int N,
                                                   __half* __restrict__ y, int ldy, int silu, float* __restrict__ xadd) {
  const int n = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (n >= N) return;
  const size_t slice = (size_t)M * N;
  for (int m = blockIdx.y; m < M; m += gridDim.y) {
    const float* p = ws + (size_t)m * N + n;
    float4 s = *reinterpret_cast<const float4*>(p);
    for (int z = 1; z < splits; z++) {
      const float4 t = *reinterpret_cast<const float4*>(p + z * slice);
      s.x += t.x, s.y += t.y, s.z += t.z, s.w += t.w;
    }
    if (xadd) {
      float4* dx = reinterpret_cast<float4*>(xadd + (size_t)m * ldy + n);
      float4 xv = *dx;
      xv.x += __half2float(__float2half_rn(s.x)), xv.y += __half2float(__float2half_rn(s.y));
      xv.z += __half2float(__float2half_rn(s.z)), xv.w += __half2float(__float2half_rn(s.w));
      *dx = xv;
    } else if (!silu) {
      const __half2 a = __floats2half2_rn(s.x, s.y), b = __floats2half2_rn(s.z, s.w);
      uint2 o;
      o.x = *reinterpret_cast<const uint32_t*>(&a);
      o.y = *reinterpret_cast<const uint32_t*>(&b);
      *reinterpret_cast<uint2*>(y + (size_t)m * ldy + n) = o;
    } else {  // columns (2j, 2j + 1) are gate and up of output j = n / 2 (and j + 1)
      *reinterpret_cast<__half2*>(y + (size_t)m * ldy + n / 2) = __floats2half2_rn(swiglu(s.x, s.y), swiglu(s.z, s.w));
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Small-M path: a weight-streaming GEMM on mma.sync for a few dozen tokens
// ---------------------------------------------------------------------------------------------
// Below about a hundred tokens the tcgen05 kernel is bound by its MMA issue (one M=128 MMA per 16 k,
// whatever N is) and by its split-K finish, not by the weight bytes (the reference switches to its
// GEMV below 21 rows for the same reason, src/engine.rs:425-431). This kernel dequantizes each
// thread's weights in registers straight into the A fragments of mma.sync.m16n8k16 (f16 in, f32
// accumulate), so nothing but the packed tile bytes moves through memory, and splits K across the
// CTAs of a thread-block cluster, which add their partial tiles through distributed shared memory in
// rank order: one launch, no workspace, the same sums run to run.
//
// A CTA of four warps takes one 128-row block of the tile layout, a range of k-tiles (one split) and
// up to 8 NT tokens. Warp w owns rows 32w .. 32w + 31 as two 16-row MMA row groups; lane (g, t) holds
// rows g, g + 8, g + 16, g + 24 of them. The MMA's k order is free (the sum over k is the same in any
// order as long as A and B agree), so in each step of two k-tiles (four 32-weight k-groups) lane t
// takes k-group t whole: one 16-byte load per row of its four 8-weight words, and word q feeds the
// two MMAs of sub-step q, whose B fragments are then the 8 activations of that word (one 16-byte
// load per token, through L1, where the CTA's four warps share them). Weights are streamed past L1.
SD_DEV uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
SD_DEV uint32_t ld_stream4(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
SD_DEV void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int kSmallThreads = 128;
constexpr int kSmallMaxSplits = 8;  // the portable cluster size
constexpr int kSmallMaxM = 256;  // tokens the small-M kernel takes (token blocks of 32 over the grid)

// Where the planner takes the small-M kernel, from steady-state times on B200 (back-to-back launches,
// weights cold; small-M vs tcgen05 tiles, us): up to 16 tokens on every shape (in_proj n = 8256:
// 10.9 vs 14.4 at m = 16, 7.2 vs 12.9 at m = 1); up to 64 tokens where the output is narrow, n <= 4096
// (down n = 2048, k = 6144: 13.3 vs 14.4 at m = 64; out_proj 2048 x 2048: 8.8 vs 10.8). The wide
// outputs past 16 tokens stay on the tcgen05 tiles (gate_up n = 12288, m = 32: 17.7 vs 15.0).
static bool small_wins(const QWeight& w, int M) { return M <= 16 || (M <= 64 && w.n <= 4096); }

// Activations: each CTA stages its tokens' k-range in chunks of 256 (two steps) through a two-chunk
// shared-memory ring (cp.async, issued with the weight loads of the chunk before), so the MMAs wait on
// shared-memory latency only. A token row of a chunk is 32 16-byte units stored at u ^ bit 3 of u, in
// rows of 34 units: a quarter warp's B loads (tokens g, g + 1; units 16 s + 4 t + q) hit 8 distinct
// bank groups.
constexpr int kSmallChunkK = 256;
constexpr int kSmallRowU = kSmallChunkK / 8 + 2;

template <int NT>
struct SmallCfg {
  static constexpr int RS = NT == 1 ? 40 : 8 * NT + 8;  // f32 row stride of the partial tile (float2 stores conflict-free)
  static constexpr int kBuf = 8 * NT * kSmallRowU * 16;  // one chunk of activations
  static constexpr int kRed = kBM * RS * 4;             // the partial tile (reuses the ring after the main loop)
  static constexpr int kSmem = 2 * kBuf > kRed ? 2 * kBuf : kRed;
};

// One step's packed weights of a lane: four rows' words of its k-group, their scale pairs (and bias pairs).
struct SmallW {
  uint4 q[4];
  uint32_t s[4], b[4];
};

template <bool ASYM>
SD_DEV void small_load(SmallW& w, const uint8_t* tile, int hb, int row0) {
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int row = row0 + 8 * r;
    w.q[r] = ld_stream16(tile + hb * kHalfCodes + row * 16);
    w.s[r] = ld_stream4(tile + kTileCodes + row * 4);
    if (ASYM) w.b[r] = ld_stream4(tile + kTileBytes + row * 4);
  }
}

SD_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Step s (0 or 1) of the chunk in `buf`: lane (g, t) reads token 8 j + g, units 16 s + 4 t + q.
template <int NT, bool ASYM>
SD_DEV void small_step(const SmallW& w, int hb, const uint4* buf, int s, int g, int t, float (&c)[2][NT][4]) {
  __half2 s2[4], b2[4];
#pragma unroll
  for (int r = 0; r < 4; r++) {
    s2[r] = __half2half2(__ushort_as_half((unsigned short)(w.s[r] >> (16 * hb))));
    if (ASYM) b2[r] = __half2half2(__ushort_as_half((unsigned short)(w.b[r] >> (16 * hb))));
  }
  const uint4* bb = buf + g * kSmallRowU + 16 * s + 4 * t;
  const int sw = t >> 1;  // bit 3 of the unit 16 s + 4 t + q
#pragma unroll
  for (int q = 0; q < 4; q++) {
    uint32_t a[2][8];
#pragma unroll
    for (int rg = 0; rg < 2; rg++) {
      const uint32_t lo = reinterpret_cast<const uint32_t*>(&w.q[2 * rg])[q];
      const uint32_t hi = reinterpret_cast<const uint32_t*>(&w.q[2 * rg + 1])[q];
#pragma unroll
      for (int p = 0; p < 4; p++) {  // element pair p of the word: k 8q + 2p, + 1 of this k-group
        __half2 vl, vh;
        if (ASYM) {
          vl = dq_pair_affine(lo, p, s2[2 * rg], b2[2 * rg]);
          vh = dq_pair_affine(hi, p, s2[2 * rg + 1], b2[2 * rg + 1]);
        } else {
          vl = dq_pair(lo, p, s2[2 * rg]);
          vh = dq_pair(hi, p, s2[2 * rg + 1]);
        }
        // A fragment: {row g, k 2t}, {row g + 8, k 2t}, {row g, k 2t + 8}, {row g + 8, k 2t + 8}; pairs 0, 1
        // are the first MMA's k 2t and 2t + 8, pairs 2, 3 the second's
        a[rg][(p >> 1) * 4 + (p & 1) * 2 + 0] = h2_as_u32(vl);
        a[rg][(p >> 1) * 4 + (p & 1) * 2 + 1] = h2_as_u32(vh);
      }
    }
#pragma unroll
    for (int j = 0; j < NT; j++) {
      const uint4 bv = bb[j * 8 * kSmallRowU + (q ^ sw)];  // (16 s + 4 t + q) ^ sw: 16 s + 4 t has its low bits clear
      mma16816(c[0][j], a[0], bv.x, bv.y);
      mma16816(c[0][j], a[0] + 4, bv.z, bv.w);
      mma16816(c[1][j], a[1], bv.x, bv.y);
      mma16816(c[1][j], a[1] + 4, bv.z, bv.w);
    }
  }
}

template <int EPI, int NT, bool ASYM>
__global__ void __launch_bounds__(kSmallThreads) gemm_q4_small(const uint8_t* __restrict__ wt, int tile_bytes, int KT,
                                                               int kts, const __half* __restrict__ act, int lda, int M,
                                                               int N, __half* __restrict__ y, int ldy,
                                                               float* __restrict__ xadd) {
  using Cfg = SmallCfg<NT>;
  constexpr int RS = Cfg::RS, TOK = 8 * NT;
  extern __shared__ __align__(16) uint8_t small_smem[];
  uint4* ring = reinterpret_cast<uint4*>(small_smem);  // [2][TOK][kSmallRowU]
  float* red = reinterpret_cast<float*>(small_smem);   // [128][RS], after the main loop
  const int S = gridDim.x, split = blockIdx.x, nb = blockIdx.y, m0 = blockIdx.z * TOK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, hb = t & 1;
  const int row0 = warp * 32 + g;
  const int kt0 = split * kts, kt1 = min(KT, kt0 + kts);
  const int nsteps = max(0, kt1 - kt0) / 2, nchunks = (nsteps + 1) / 2;
  // lane t's k-group in step i: k-tile kt0 + 2 i + t / 2, half t % 2
  const uint8_t* tile0 = wt + ((size_t)nb * KT + kt0 + (t >> 1)) * tile_bytes;
  const size_t step_bytes = (size_t)2 * tile_bytes;
  const int ntok = min(TOK, M - m0);
  const int k0 = kt0 * kBK, kend = kt1 * kBK;

  float c[2][NT][4];
#pragma unroll
  for (int rg = 0; rg < 2; rg++)
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) c[rg][j][e] = 0.0f;

  // the weights depend on nothing the stream computes: the first two steps' loads go out before the
  // wait for the kernel before (programmatic dependent launch)
  SmallW w0, w1;
  if (nsteps > 0) small_load<ASYM>(w0, tile0, hb, row0);
  if (nsteps > 1) small_load<ASYM>(w1, tile0 + step_bytes, hb, row0);
  grid_dep_wait();
  // chunk ch of the activations into ring slot ch % 2 (tokens past M and k past the split stay unloaded:
  // they only reach output columns that are never stored, or no product at all)
  auto load_chunk = [&](int ch) {
    uint4* dst = ring + (ch & 1) * TOK * kSmallRowU;
    const int kc = k0 + ch * kSmallChunkK;
    for (int idx = threadIdx.x; idx < TOK * (kSmallChunkK / 8); idx += kSmallThreads) {
      const int tk = idx / (kSmallChunkK / 8), u = idx % (kSmallChunkK / 8);
      if (tk < ntok && kc + 8 * u < kend)
        cp_async16(dst + tk * kSmallRowU + (u ^ ((u >> 3) & 1)), act + (size_t)(m0 + tk) * lda + kc + 8 * u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (nchunks > 0) load_chunk(0);
#pragma unroll 1
  for (int ch = 0; ch < nchunks; ch++) {
    if (ch + 1 < nchunks) {
      load_chunk(ch + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint4* buf = ring + (ch & 1) * TOK * kSmallRowU;
    const int i = 2 * ch;
    small_step<NT, ASYM>(w0, hb, buf, 0, g, t, c);
    if (i + 2 < nsteps) small_load<ASYM>(w0, tile0 + (i + 2) * step_bytes, hb, row0);
    if (i + 1 < nsteps) {
      small_step<NT, ASYM>(w1, hb, buf, 1, g, t, c);
      if (i + 3 < nsteps) small_load<ASYM>(w1, tile0 + (i + 3) * step_bytes, hb, row0);
    }
    __syncthreads();  // the slot is loaded again two chunks on
  }

  // the partial tile: C fragment {row g, tokens 2t, 2t + 1}, {row g + 8, same}
#pragma unroll
  for (int rg = 0; rg < 2; rg++)
#pragma unroll
    for (int j = 0; j < NT; j++) {
      const int r = warp * 32 + rg * 16 + g, col = 8 * j + 2 * t;
      *reinterpret_cast<float2*>(&red[r * RS + col]) = make_float2(c[rg][j][0], c[rg][j][1]);
      *reinterpret_cast<float2*>(&red[(r + 8) * RS + col]) = make_float2(c[rg][j][2], c[rg][j][3]);
    }
  cg::cluster_group cluster = cg::this_cluster();
  if (S > 1) cluster.sync();
  else __syncthreads();

  // rank r finishes rows [r 128 / S, (r + 1) 128 / S): the splits' partials summed in rank order
  const float* part[kSmallMaxSplits];
#pragma unroll
  for (int sp = 0; sp < kSmallMaxSplits; sp++) part[sp] = sp < S ? (S > 1 ? cluster.map_shared_rank(red, sp) : red) : red;
  const int rows = kBM / S, rb = (S > 1 ? (int)cluster.block_rank() : 0) * rows;
  const int n0 = nb * kBM;
  for (int e = threadIdx.x; e < (rows / 2) * ntok; e += kSmallThreads) {
    const int rp = e % (rows / 2), tk = e / (rows / 2);
    const int r = rb + 2 * rp, n = n0 + r;
    float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
    for (int sp = 0; sp < kSmallMaxSplits; sp++)
      if (sp < S) {
        v0 += part[sp][r * RS + tk];
        v1 += part[sp][(r + 1) * RS + tk];
      }
    if (n >= N) continue;  // N is even: rows n and n + 1 are both in or both out
    const size_t o = (size_t)(m0 + tk) * ldy;
    if (EPI == kEpiSilu) {
      y[o + n / 2] = __float2half_rn(swiglu(v0, v1));
    } else if (EPI == kEpiAdd) {
      float2* px = reinterpret_cast<float2*>(xadd + o + n);
      float2 xv = *px;
      xv.x += __half2float(__float2half_rn(v0));
      xv.y += __half2float(__float2half_rn(v1));
      *px = xv;
    } else {
      *reinterpret_cast<__half2*>(y + o + n) = __floats2half2_rn(v0, v1);
    }
  }
  if (S > 1) cluster.sync();  // no CTA leaves while another still reads its partial tile
}

// Reference layout -> tile layout. The reference stores each row as k/32 blocks of 32 codes of `bits`
// bits (src/kernels.rs:545-586: int4 as 4 words of 8 nibbles; int2 as 2 words of 16 two-bit fields;
// int3 as those 2 words for the low two bits and a third word for the high bits) with one f16 scale
// per `group` weights, taken by the global block index (row * k/32 + block) / (group / 32). A
// symmetric code q means (q - 2^(bits-1)) * scale; as the int4 code q + 8 - 2^(bits-1) (0..15) it means
// the same value under the int4 rule (code - 8) * scale, and each 32-block gets its own copy of its
// group's scale, so every symmetric format becomes the GEMM's one format without changing a value.
// Tile layout: [npad/128][k/64][2048 code bytes of k-group 0 (16 per row) + 2048 of k-group 1 + 512
// scale bytes (2 per row)], so that 32 consecutive rows read by a warp are contiguous, with the nibbles
// of each 8-element word reordered to (even elements low half, odd elements high half). `interleave`
// maps output row 2j to source row j and 2j+1 to source row n/2 + j (gate_up: gate j next to up j).
SD_DEV uint32_t code_at(const uint8_t* blk, int bits, int e) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(blk);
  if (bits == 4) return (w[e >> 3] >> (4 * (e & 7))) & 15u;
  uint32_t c = (w[e >> 4] >> (2 * (e & 15))) & 3u;
  if (bits == 3) c |= ((w[2] >> e) & 1u) << 2;
  return c;
}
__global__ void repack_q4(const uint8_t* __restrict__ q, const __half* __restrict__ s, const __half* __restrict__ b, int n, int k,
                          int npad, int interleave, int bits, int group, uint8_t* __restrict__ out) {
  const int KT = k / kBK, nb = k / 32, bb = 4 * bits, gpb = group / 32;
  const int tb = b ? kTileBytesMax : kTileBytes;
  const uint32_t shift = b ? 0u : 8u - (1u << (bits - 1));  // asymmetric codes stay as they are
  const int64_t total = (int64_t)npad * KT;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(idx / KT), kt = (int)(idx % KT);
    int src = row;
    if (interleave) src = (row & 1) ? (n / 2 + (row >> 1)) : (row >> 1);
    uint8_t* tile = out + ((size_t)(row / kBM) * KT + kt) * tb;
    uint32_t* dst0 = reinterpret_cast<uint32_t*>(tile + (row % kBM) * 16);               // k-group 0
    uint32_t* dst1 = reinterpret_cast<uint32_t*>(tile + kHalfCodes + (row % kBM) * 16);  // k-group 1
    __half* dsc = reinterpret_cast<__half*>(tile + kTileCodes) + (row % kBM) * 2;
    __half* dbi = reinterpret_cast<__half*>(tile + kTileBytes) + (row % kBM) * 2;  // asymmetric only
    if (row >= n) {
      for (int i = 0; i < 4; i++) dst0[i] = dst1[i] = 0;
      dsc[0] = dsc[1] = __float2half(0.0f);
      if (b) dbi[0] = dbi[1] = __float2half(0.0f);
      continue;
    }
    for (int hb = 0; hb < 2; hb++) {  // the two 32-blocks of this k-tile
      const size_t blk = (size_t)src * nb + 2 * kt + hb;
      const uint8_t* bp = q + blk * bb;
      for (int i = 0; i < 4; i++) {
        uint32_t o = 0;
        for (int e = 0; e < 8; e++) {
          const uint32_t c4 = code_at(bp, bits, 8 * i + e) + shift;
          const int pos = (e & 1) ? (4 + (e >> 1)) : (e >> 1);
          o |= c4 << (4 * pos);
        }
        (hb ? dst1 : dst0)[i] = o;
      }
      dsc[hb] = s[blk / gpb];
      if (b) dbi[hb] = b[blk / gpb];
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// A 2D f16 tensor map over rows x cols (row-major, row stride ld elements), box {64, box_rows},
// 128-byte swizzle, zero fill out of bounds.
int make_act_map(CUtensorMap* map, const void* ptr, int rows, int cols, int ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// A 3-D f16 tensor map [z][y][x] (x contiguous, y rows `ystride` elements apart, z slabs `zstride`
// elements apart; dims x, y, z) with boxes of 64 x box_y x 1 and the 128-byte swizzle. Coordinates
// outside the dims read zeros.
int make_map_3d(CUtensorMap* map, const void* ptr, int x, int y, int z, long long ystride, long long zstride, int box_y) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[3] = {(cuuint64_t)x, (cuuint64_t)y, (cuuint64_t)z};
  cuuint64_t strides[2] = {(cuuint64_t)ystride * 2, (cuuint64_t)zstride * 2};
  cuuint32_t box[3] = {64u, (cuuint32_t)box_y, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// A 2-D f32 tensor map over rows x cols (row-major, rows `ld` elements apart) with boxes of
// 32 x box_rows and the 128-byte swizzle (a box row is one 128-byte line). Stores clip at the dims.
int make_map_f32(CUtensorMap* map, const void* ptr, long long rows, int cols, long long ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {32u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

template <int BN, int EPI>
static cudaError_t launch_bn(const CUtensorMap& map, const QWeight& w, int M, const TileGrid& tg, int num_sms, __half* y,
                             int ldy, float* ws, int* err, cudaStream_t st) {
  using Cfg = CfgOf<BN, EPI>;
  auto kern = gemm_q4_tc<BN, EPI>;
  static std::atomic<bool> attr_set[kMaxDevices] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  // launched as a programmatic dependent of the kernel before it: its set-up (barriers, TMEM, the
  // weight tiles' first copies, which depend on nothing the stream computes) overlaps that kernel's
  // tail; the activation loads and the epilogue wait for it (grid_dep_wait)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(tg.count(), num_sms));
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, map, (const uint8_t*)w.tiles, M, w.n, w.tile_bytes, tg, y, ldy, ws, err);
}

template <int EPI>
static cudaError_t launch_epi(int bn, const CUtensorMap& map, const QWeight& w, int M, const TileGrid& tg, int num_sms,
                              __half* y, int ldy, float* ws, int* err, cudaStream_t st) {
  switch (bn) {
    case 32: return launch_bn<32, EPI>(map, w, M, tg, num_sms, y, ldy, ws, err, st);
    case 64: return launch_bn<64, EPI>(map, w, M, tg, num_sms, y, ldy, ws, err, st);
    case 128: return launch_bn<128, EPI>(map, w, M, tg, num_sms, y, ldy, ws, err, st);
    default: return launch_bn<192, EPI>(map, w, M, tg, num_sms, y, ldy, ws, err, st);
  }
}

// Token tile width and split-K, from a time estimate: (waves of work units over the SMs) x (k-tiles
// per unit) x the steady-state time of a k-tile at that width (measured on B200 with one full wave of
// 128-row weight tiles: 0.33 us at 32 or 64 tokens, 0.35 us at 128, 0.385 us at 192), plus, with K
// split, the finishing pass: a launch and the f32 partials written and read back (8 bytes per output
// per split at about 5 TB/s). Past 128 tokens both 128- and 192-wide tiles are costed (192 does more
// per k-tile, 128 can fill the last wave better).
static int split_kps(int KT, int splits) {  // k-tiles per split: even where K allows (two-k-tile stages)
  int kps = (KT + splits - 1) / splits;
  if (KT % 2 == 0) kps += kps & 1;
  return kps;
}

static double kt_us(int bn) { return bn >= 192 ? 0.385 : (bn >= 128 ? 0.35 : 0.33); }

void gemm_plan(const QWeight& w, int M, int num_sms, int* bn_out, int* splits_out, int* kps_out) {
  const int ntiles = w.npad / kBM;
  const int KT = w.k / kBK;
  int cands[2] = {M <= 32 ? 32 : (M <= 64 ? 64 : 128), 0};
  if (M > 128) cands[1] = 192;
  double best_cost = 1e30;
  int best_bn = cands[0], best_s = 1;
  for (int bn : cands) {
    if (!bn) continue;
    const long tiles = (long)ntiles * ((M + bn - 1) / bn);
    for (int s = 1; s <= std::max(1, KT / 4); s++) {  // at least 4 k-tiles per split
      const int kps = split_kps(KT, s);
      if ((KT + kps - 1) / kps != s) continue;
      const long waves = (tiles * s + num_sms - 1) / num_sms;
      double cost = waves * kps * kt_us(bn);
      if (s > 1) cost += 3.0 + (double)s * M * w.n * 8.0 / 5e6;
      if (cost < best_cost) best_cost = cost, best_bn = bn, best_s = s;
    }
  }
  *bn_out = best_bn;
  *splits_out = best_s;
  *kps_out = split_kps(KT, best_s);
}

// Tile order from the HBM traffic it implies: an operand that does not fit in (a share of) L2 is read
// from HBM once per tile of the other operand's axis unless its own tiles are the outer loop. The
// share is a quarter of the 126 MB L2 (each die's half holds the lines it reads fastest): on B200 at
// M = 16384 the token-major order measured 1122 vs 849 TFLOP/s (down, K = 6144: 201 MB of
// activations) and 1124 vs 1036 (gate_up, K = 2048: 67 MB), and the same at M = 1536.
bool gemm_token_major(const QWeight& w, int M) {
  constexpr double kL2 = 32e6;  // bytes of L2 an operand may occupy and still be re-read from L2
  const double act = (double)M * w.k * 2, wts = (double)w.bytes;
  const double ntiles = w.npad / kBM, mtiles = (M + 191) / 192;
  const double weight_major = wts + (act > kL2 ? act * ntiles : act);
  const double token_major = act + (wts > kL2 ? wts * mtiles : wts);
  return token_major < weight_major;
}

// The small-M kernel's shape: NT token groups of 8 per CTA (the fewest that hold M, up to 32 tokens, then
// CTAs over token blocks of 32), and K split in k-tile pairs over a cluster of up to 8 CTAs until
// about two CTAs per SM are busy. False where it does not apply (K not a multiple of 128). Measured on
// B200 (back-to-back launches, weights cold): 32-token blocks beat 64-token ones at every shape (the
// MMAs are latency-bound at one warp per SM quarter: in_proj m = 64, 26.9 -> 21.2 us; down 18.7 ->
// 13.3 us), and splitting to two CTAs per SM beat one and four on the wide shapes.
bool gemm_small_plan(const QWeight& w, int M, int num_sms, int* nt_out, int* splits_out, int* kts_out) {
  const int KT = w.k / kBK;
  if (KT % 2 || M <= 0 || M > kSmallMaxM) return false;
  const int nt = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  const long ctas = (long)(w.npad / kBM) * ((M + 8 * nt - 1) / (8 * nt));
  const int steps = KT / 2;
  int s = 1;
  while (s < kSmallMaxSplits && 2 * s <= steps && s * ctas < 2L * num_sms) s *= 2;
  *nt_out = nt;
  *splits_out = s;
  *kts_out = 2 * ((steps + s - 1) / s);
  return true;
}

template <int EPI, int NT, bool ASYM>
static cudaError_t launch_small(const QWeight& w, const __half* act, int lda, int M, int S, int kts, __half* y, int ldy,
                                float* xadd, cudaStream_t st) {
  auto kern = gemm_q4_small<EPI, NT, ASYM>;
  static std::atomic<bool> attr_set[kMaxDevices] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_set[dev].load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SmallCfg<NT>::kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, w.npad / kBM, (M + 8 * NT - 1) / (8 * NT));
  cfg.blockDim = dim3(kSmallThreads);
  cfg.dynamicSmemBytes = SmallCfg<NT>::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = S;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = S > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, (const uint8_t*)w.tiles, w.tile_bytes, w.k / kBK, kts, act,
                            lda, M, w.n, y, ldy, xadd);
}

template <int EPI, bool ASYM>
static cudaError_t launch_small_nt(int nt, const QWeight& w, const __half* act, int lda, int M, int S, int kts, __half* y,
                                   int ldy, float* xadd, cudaStream_t st) {
  switch (nt) {
    case 1: return launch_small<EPI, 1, ASYM>(w, act, lda, M, S, kts, y, ldy, xadd, st);
    case 2: return launch_small<EPI, 2, ASYM>(w, act, lda, M, S, kts, y, ldy, xadd, st);
    default: return launch_small<EPI, 4, ASYM>(w, act, lda, M, S, kts, y, ldy, xadd, st);
  }
}

template <int EPI>
static cudaError_t launch_small_epi(int nt, const QWeight& w, const __half* act, int lda, int M, int S, int kts, __half* y,
                                    int ldy, float* xadd, cudaStream_t st) {
  return w.asym ? launch_small_nt<EPI, true>(nt, w, act, lda, M, S, kts, y, ldy, xadd, st)
                : launch_small_nt<EPI, false>(nt, w, act, lda, M, S, kts, y, ldy, xadd, st);
}

cudaError_t gemm_q4(const QWeight& w, const __half* act, int M, int lda, __half* y, int ldy, bool silu, float* ws,
                    size_t ws_bytes, int* err, int num_sms, cudaStream_t st, int* nlaunch, float* xadd, int algo) {
  if (nlaunch) *nlaunch = 0;
  if (M <= 0) return cudaSuccess;
  if (xadd && (silu || w.n % 4 || ldy % 4 || (uintptr_t)xadd % 16)) return cudaErrorInvalidValue;
  int nt, ssplits, kts;
  if (algo != 1 && gemm_small_plan(w, M, num_sms, &nt, &ssplits, &kts) && (algo == 2 || small_wins(w, M)) &&
      lda % 8 == 0 && (uintptr_t)act % 16 == 0) {
    if (nlaunch) *nlaunch = 1;
    return xadd ? launch_small_epi<kEpiAdd>(nt, w, act, lda, M, ssplits, kts, nullptr, ldy, xadd, st)
                : silu ? launch_small_epi<kEpiSilu>(nt, w, act, lda, M, ssplits, kts, y, ldy, nullptr, st)
                       : launch_small_epi<kEpiStore>(nt, w, act, lda, M, ssplits, kts, y, ldy, nullptr, st);
  }
  if (algo == 2) return cudaErrorInvalidValue;  // the small-M kernel does not take this shape
  int bn, splits, kps;
  gemm_plan(w, M, num_sms, &bn, &splits, &kps);
  const int KT = w.k / kBK;
  const size_t slice = (size_t)M * w.n * sizeof(float);
  if (splits > 1 && splits * slice > ws_bytes) {  // fewer splits that fit the workspace
    const int fit = (int)std::min<size_t>(splits, ws_bytes / std::max<size_t>(slice, 1));
    splits = std::max(1, fit);
    kps = split_kps(KT, splits);
    splits = (KT + kps - 1) / kps;
    if (splits * slice > ws_bytes) splits = 1, kps = KT;
  }
  if (w.n % 4) splits = 1, kps = KT;  // the finish reads four partial columns at a time
  CUtensorMap map;
  if (make_act_map(&map, act, M, w.k, lda, bn) != 0) return cudaErrorInvalidValue;
  TileGrid tg{w.npad / kBM, (M + bn - 1) / bn, splits, kps, KT, gemm_token_major(w, M) ? 1 : 0};
  if (nlaunch) *nlaunch = splits == 1 ? 1 : 2;
  if (splits == 1)
    return xadd ? launch_epi<kEpiAdd>(bn, map, w, M, tg, num_sms, nullptr, ldy, xadd, err, st)
                : silu ? launch_epi<kEpiSilu>(bn, map, w, M, tg, num_sms, y, ldy, nullptr, err, st)
                       : launch_epi<kEpiStore>(bn, map, w, M, tg, num_sms, y, ldy, nullptr, err, st);
  cudaError_t e = launch_epi<kEpiPartial>(bn, map, w, M, tg, num_sms, y, ldy, ws, err, st);
  if (e != cudaSuccess) return e;
  const dim3 grid((w.n / 4 + 255) / 256, std::min(M, 65535));
  gemm_finish<<<grid, 256, 0, st>>>(ws, splits, M, w.n, y, ldy, silu ? 1 : 0, xadd);
  return cudaGetLastError();
}

template <int BN>
static cudaError_t preload_bn() {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(gemm_q4_tc<BN, kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)CfgOf<BN, kEpiStore>::kSmem)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(gemm_q4_tc<BN, kEpiSilu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)CfgOf<BN, kEpiSilu>::kSmem)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(gemm_q4_tc<BN, kEpiAdd>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)CfgOf<BN, kEpiAdd>::kSmem)) != cudaSuccess)
    return e;
  return cudaFuncSetAttribute(gemm_q4_tc<BN, kEpiPartial>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)CfgOf<BN, kEpiPartial>::kSmem);
}

// Loads every GEMM kernel on the current device (and sets its shared-memory size), so that no launch
// later pays the first-use module load.
cudaError_t preload_gemm() {
  cudaError_t e;
  if ((e = preload_bn<32>()) != cudaSuccess || (e = preload_bn<64>()) != cudaSuccess || (e = preload_bn<128>()) != cudaSuccess ||
      (e = preload_bn<192>()) != cudaSuccess)
    return e;
  cudaFuncAttributes a;
  const void* small[] = {
      (const void*)gemm_q4_small<kEpiStore, 1, false>, (const void*)gemm_q4_small<kEpiStore, 2, false>,
      (const void*)gemm_q4_small<kEpiStore, 4, false>, (const void*)gemm_q4_small<kEpiSilu, 1, false>,
      (const void*)gemm_q4_small<kEpiSilu, 2, false>,  (const void*)gemm_q4_small<kEpiSilu, 4, false>,
      (const void*)gemm_q4_small<kEpiAdd, 1, false>,   (const void*)gemm_q4_small<kEpiAdd, 2, false>,
      (const void*)gemm_q4_small<kEpiAdd, 4, false>,   (const void*)gemm_q4_small<kEpiStore, 1, true>,
      (const void*)gemm_q4_small<kEpiStore, 2, true>,  (const void*)gemm_q4_small<kEpiStore, 4, true>,
      (const void*)gemm_q4_small<kEpiSilu, 1, true>,   (const void*)gemm_q4_small<kEpiSilu, 2, true>,
      (const void*)gemm_q4_small<kEpiSilu, 4, true>,   (const void*)gemm_q4_small<kEpiAdd, 1, true>,
      (const void*)gemm_q4_small<kEpiAdd, 2, true>,    (const void*)gemm_q4_small<kEpiAdd, 4, true>};
  for (const void* f : small)
    if ((e = cudaFuncGetAttributes(&a, f)) != cudaSuccess) return e;
  if ((e = cudaFuncGetAttributes(&a, gemm_finish)) != cudaSuccess) return e;
  return cudaFuncGetAttributes(&a, repack_q4);
}

cudaError_t repack_weight(const uint8_t* q, const __half* s, int n, int k, bool interleave, QWeight* out, cudaStream_t st,
                          int bits, int group, const __half* b) {
  if ((bits != 2 && bits != 3 && bits != 4) || group < 32 || group % 32) return cudaErrorInvalidValue;
  out->n = n;
  out->k = k;
  out->npad = (n + kBM - 1) / kBM * kBM;
  out->interleaved = interleave;
  out->asym = b != nullptr;
  out->tile_bytes = b ? kTileBytesMax : kTileBytes;
  const size_t bytes = (size_t)(out->npad / kBM) * (k / kBK) * out->tile_bytes;
  cudaError_t e = cudaMalloc(&out->tiles, bytes);
  if (e != cudaSuccess) return e;
  out->bytes = bytes;
  const int64_t total = (int64_t)out->npad * (k / kBK);
  repack_q4<<<(int)std::min<int64_t>((total + 255) / 256, 8192), 256, 0, st>>>(q, s, b, n, k, out->npad, interleave ? 1 : 0, bits,
                                                                               group, out->tiles);
  return cudaGetLastError();
}

}  // namespace sd
