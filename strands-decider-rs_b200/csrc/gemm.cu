// Dequantizing GEMM on the 5th-generation tensor cores: Y[m][n] = sum_k A[m][k] W[n][k], with W
// stored as the reference's int4 group-32 symmetric blocks (src/kernels.rs:545-576, `matmul_tiled`
// at src/kernels.rs:640-709 and `matmul_coop` at :716-804 are the kernels it replaces).
//
// Roles (6 warps): warp 0 issues the TMA load of each activation tile and the bulk copy of each
// packed weight tile; warp 1 owns the TMEM accumulator and issues tcgen05.mma; warps 2-5 dequantize
// the packed weight tile into a 128-byte-swizzled f16 tile (the MMA's A operand), then run the
// epilogue out of TMEM. The weights are the MMA's M side (128 rows per tile) and the tokens its N
// side (BN columns), so one dequantized tile serves up to 256 tokens.
//
// Numerics: the dequantized weight is (q - 8) * scale rounded to f16, as the reference's tiled
// kernel computes it (src/kernels.rs:671); products accumulate in f32; the output is rounded to f16.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "sd_internal.h"

namespace sd {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kTileCodes = kBM * kBK / 2;          // 4096 bytes of int4 codes
constexpr int kTileScales = kBM * (kBK / 32) * 2;  // 512 bytes of f16 scales
constexpr int kTileBytes = kTileCodes + kTileScales;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN >= 256 ? 4 : (BN >= 128 ? 5 : (BN >= 64 ? 7 : 8));
  static constexpr int kAccCols = BN < 32 ? 32 : BN;  // one accumulator buffer
  static constexpr int kTmemCols = 2 * kAccCols;      // double-buffered: epilogue overlaps the next tile
  static constexpr size_t kA = (size_t)kBM * kBK * 2;
  static constexpr size_t kB = (size_t)BN * kBK * 2;
  static constexpr size_t kOffB = kStages * kA;
  static constexpr size_t kOffRaw = kOffB + kStages * kB;
  static constexpr size_t kOffStage = kOffRaw + (size_t)kStages * kTileBytes;
  static constexpr int kStageBytesPerWarp = 32 * 40 * 2;  // 32 x 32 f16 (row stride 40) or 16 x 32 f32 (row stride 36)
  static constexpr size_t kOffBar = kOffStage + 4 * kStageBytesPerWarp;
  static constexpr size_t kBytes = kOffBar + (3 * kStages + 4) * 8 + 16;
  static constexpr size_t kSmem = kBytes + 1024;  // room to align the base to 1024 bytes
  static_assert(kSmem <= 232448, "shared memory per CTA");
};

enum Epi { kEpiStore = 0, kEpiSilu = 1, kEpiPartial = 2 };

constexpr int kGemmThreads = 448;  // 14 warps: producer, MMA, 8 dequant, 4 epilogue

struct TileGrid {
  int ntiles, mtiles, splits, kps, KT;
  __host__ __device__ int count() const { return ntiles * mtiles * splits; }
  // consecutive tiles share the weight tile (same n-tile, all m-tiles and splits next to each other)
  __device__ void decode(int t, int& nt, int& mt, int& sp, int& kt0, int& nk) const {
    nt = t / (mtiles * splits);
    const int r = t % (mtiles * splits);
    mt = r / splits;
    sp = r % splits;
    kt0 = sp * kps;
    nk = max(0, min(KT, kt0 + kps) - kt0);
  }
};

// Persistent, warp-specialised: each CTA walks tiles blockIdx.x, +gridDim.x, ...; the smem ring runs
// across tile boundaries and the accumulator is double-buffered in TMEM, so one tile's epilogue
// overlaps the next tile's loads, dequantization and MMAs.
template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_q4_tc(const __grid_constant__ CUtensorMap act_map, const uint8_t* __restrict__ wt, int M, int N, TileGrid tg,
               __half* __restrict__ y, int ldy, float* __restrict__ ws, int* err) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = base;
  uint8_t* sb = base + Cfg::kOffB;
  uint8_t* sraw = base + Cfg::kOffRaw;
  uint8_t* sstage = base + Cfg::kOffStage;
  uint64_t* full_raw = reinterpret_cast<uint64_t*>(base + Cfg::kOffBar);
  uint64_t* full_a = full_raw + S;
  uint64_t* empty = full_a + S;
  uint64_t* acc_full = empty + S;  // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntile_total = tg.count();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&full_a[s], 256);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int KT = tg.KT;

  if (warp == 0) {
    // producer: activation tile by TMA, packed weight tile by bulk copy, one stage per k-tile
    if (lane == 0) {
      prefetch_tmap(&act_map);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x) {
        int nt, mt, sp, kt0, nk;
        tg.decode(t, nt, mt, sp, kt0, nk);
        const uint8_t* wtile = wt + (size_t)nt * KT * kTileBytes;
        for (int i = 0; i < nk; i++, it++) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (it >= S && !mbar_wait(&empty[s], ph ^ 1, abort, err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_raw[s], (uint32_t)(Cfg::kB + kTileBytes));
          tma_load_2d(sb + s * Cfg::kB, &act_map, &full_raw[s], (kt0 + i) * kBK, mt * BN);
          bulk_load(sraw + s * kTileBytes, wtile + (size_t)(kt0 + i) * kTileBytes, kTileBytes, &full_raw[s]);
        }
      }
    }
  } else if (warp == 1) {
    // MMA issuer: accumulator buffer (local tile index & 1)
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kBM, BN);
      int it = 0, lt = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x) {
        int nt, mt, sp, kt0, nk;
        tg.decode(t, nt, mt, sp, kt0, nk);
        if (nk == 0) continue;
        lt++;  // tiles with work, in order: the accumulator buffer is lt & 1
        const int buf = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, abort, err, kErrTimeoutEmpty)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * Cfg::kAccCols;
        for (int i = 0; i < nk; i++, it++) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&full_a[s], ph, abort, err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_desc(sa + s * Cfg::kA);
          const uint64_t bd = sw128_desc(sb + s * Cfg::kB);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++)  // 16 f16 = 32 bytes per step: +2 in the address field
            tc_mma_f16(acc, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0);
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full[buf]);
      }
    }
  } else if (warp < 10) {
    // dequantization: 256 threads, thread pair (r, r + 128) splits row r's 8 chunks 4 + 4
    const int tid = threadIdx.x - 64;
    const int r = tid & 127, half = tid >> 7;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x) {
      int nt, mt, sp, kt0, nk;
      tg.decode(t, nt, mt, sp, kt0, nk);
      for (int i = 0; i < nk; i++, it++) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&full_raw[s], ph, abort, err, kErrTimeoutFull)) {
          ok = false;
          break;
        }
        const uint8_t* raw = sraw + s * kTileBytes;
        const uint4 c = *reinterpret_cast<const uint4*>(raw + r * 32 + half * 16);
        const __half sc = reinterpret_cast<const __half*>(raw + kTileCodes)[r * 2 + half];
        const __half2 sc2 = __half2half2(sc);
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        uint8_t* arow = sa + s * Cfg::kA + r * 128;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int ch = half * 4 + j;
          uint4 o;
          o.x = h2_as_u32(dq_pair(w[j], 0, sc2));
          o.y = h2_as_u32(dq_pair(w[j], 1, sc2));
          o.z = h2_as_u32(dq_pair(w[j], 2, sc2));
          o.w = h2_as_u32(dq_pair(w[j], 3, sc2));
          *reinterpret_cast<uint4*>(arow + ((ch ^ (r & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();
        mbar_arrive(&full_a[s]);
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (weight rows of the tile), transposes
    // through shared memory and stores token rows with 16-byte stores
    const int q = warp & 3;
    uint8_t* stg = sstage + (warp - 10) * Cfg::kStageBytesPerWarp;
    int lt = -1;
    for (int t = blockIdx.x; t < ntile_total; t += gridDim.x) {
      int nt, mt, sp, kt0, nk;
      tg.decode(t, nt, mt, sp, kt0, nk);
      if (nk == 0) continue;
      lt++;
      const int buf = lt & 1;
      if (!mbar_wait(&acc_full[buf], (lt >> 1) & 1, abort, err, kErrTimeoutAccum)) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * Cfg::kAccCols + ((uint32_t)(q * 32) << 16);
      const int n0 = nt * kBM + q * 32;  // first weight row of this warp
      if (EPI != kEpiPartial) {
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
            // rows interleaved as (gate j, up j): even lanes hold gate, odd lanes up
#pragma unroll
            for (int j = 0; j < 32; j++) {
              const float g = __half2float(__float2half_rn(__uint_as_float(v[j])));
              const float u = __shfl_xor_sync(0xffffffffu, g, 1);
              if ((lane & 1) == 0) st[j * 40 + (lane >> 1)] = __float2half_rn(g / (1.0f + __expf(-g)) * u);
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
      mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// Split-K finish: sums the splits' f32 partials in split order (deterministic), then f16 (or the
// SwiGLU of interleaved gate/up rows).
__global__ void gemm_finish(const float* __restrict__ ws, int splits, int M, int N, __half* __restrict__ y, int ldy, int silu) {
  const int64_t total = silu ? (int64_t)M * (N / 2) : (int64_t)M * N;
  const int64_t slice = (int64_t)M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    if (!silu) {
      const int64_t m = i / N, n = i % N;
      float s = 0.0f;
      for (int z = 0; z < splits; z++) s += ws[z * slice + i];
      y[m * ldy + n] = __float2half_rn(s);
    } else {
      const int64_t half = N / 2, m = i / half, j = i % half;
      float gs = 0.0f, us = 0.0f;
      for (int z = 0; z < splits; z++) {
        gs += ws[z * slice + m * N + 2 * j];
        us += ws[z * slice + m * N + 2 * j + 1];
      }
      const float g = __half2float(__float2half_rn(gs));
      const float u = __half2float(__float2half_rn(us));
      y[m * ldy + j] = __float2half_rn(g / (1.0f + __expf(-g)) * u);
    }
  }
}

// Reference layout (n rows of k/32 blocks of 16 bytes; scales [n][k/32]) -> tile layout
// [npad/128][k/64][4096 code bytes + 512 scale bytes], with the nibbles of each 8-element word
// reordered to (even elements low half, odd elements high half). `interleave` maps output row 2j
// to source row j and 2j+1 to source row n/2 + j (gate_up: gate j next to up j).
__global__ void repack_q4(const uint8_t* __restrict__ q, const __half* __restrict__ s, int n, int k, int npad, int interleave,
                          uint8_t* __restrict__ out) {
  const int KT = k / kBK;
  const int64_t total = (int64_t)npad * KT;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(idx / KT), kt = (int)(idx % KT);
    int src = row;
    if (interleave) src = (row & 1) ? (n / 2 + (row >> 1)) : (row >> 1);
    uint8_t* tile = out + ((size_t)(row / kBM) * KT + kt) * kTileBytes;
    uint32_t* dst = reinterpret_cast<uint32_t*>(tile + (row % kBM) * 32);
    __half* dsc = reinterpret_cast<__half*>(tile + kTileCodes) + (row % kBM) * 2;
    if (row >= n) {
      for (int i = 0; i < 8; i++) dst[i] = 0;
      dsc[0] = dsc[1] = __float2half(0.0f);
      continue;
    }
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(q + ((size_t)src * (k / 32) + 2 * kt) * 16);
    for (int i = 0; i < 8; i++) {
      const uint32_t w = sw[i];
      uint32_t o = 0;
      for (int e = 0; e < 8; e++) {
        const uint32_t nib = (w >> (4 * e)) & 15u;
        const int pos = (e & 1) ? (4 + (e >> 1)) : (e >> 1);
        o |= nib << (4 * pos);
      }
      dst[i] = o;
    }
    dsc[0] = s[(size_t)src * (k / 32) + 2 * kt];
    dsc[1] = s[(size_t)src * (k / 32) + 2 * kt + 1];
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

template <int BN, int EPI>
static cudaError_t launch_bn(const CUtensorMap& map, const QWeight& w, int M, const TileGrid& tg, int num_sms, __half* y,
                             int ldy, float* ws, int* err, cudaStream_t st) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_q4_tc<BN, EPI>;
  static bool attr_set[kMaxDevices] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int grid = std::min(tg.count(), num_sms);
  kern<<<grid, kGemmThreads, Cfg::kSmem, st>>>(map, w.tiles, M, w.n, tg, y, ldy, ws, err);
  return cudaGetLastError();
}

template <int EPI>
static cudaError_t launch_epi(int bn, const CUtensorMap& map, const QWeight& w, int M, const TileGrid& tg, int num_sms,
                              __half* y, int ldy, float* ws, int* err, cudaStream_t st) {
  switch (bn) {
    case 32: return launch_bn<32, EPI>(map, w, M, tg, num_sms, y, ldy, ws, err, st);
    case 64: return launch_bn<64, EPI>(map, w, M, tg, num_sms, y, ldy, ws, err, st);
    case 128: return launch_bn<128, EPI>(map, w, M, tg, num_sms, y, ldy, ws, err, st);
    default: return launch_bn<256, EPI>(map, w, M, tg, num_sms, y, ldy, ws, err, st);
  }
}

// Token tile width and split-K: 256-wide token tiles for long prompts, narrower ones (with the K
// dimension split across CTAs) when the weight tiles alone would leave most SMs idle.
void gemm_plan(const QWeight& w, int M, int num_sms, int* bn_out, int* splits_out, int* kps_out) {
  int bn = M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256));
  const int ntiles = w.npad / kBM;
  const int mtiles = (M + bn - 1) / bn;
  const int KT = w.k / kBK;
  int splits = 1;
  const int tiles = ntiles * mtiles;
  if (tiles < num_sms) {
    splits = (num_sms + tiles - 1) / tiles;
    splits = std::min(splits, std::max(1, KT / 4));  // at least 4 k-tiles per split
  }
  const int kps = (KT + splits - 1) / splits;
  splits = (KT + kps - 1) / kps;
  *bn_out = bn;
  *splits_out = splits;
  *kps_out = kps;
}

cudaError_t gemm_q4(const QWeight& w, const __half* act, int M, int lda, __half* y, int ldy, bool silu, float* ws,
                    size_t ws_bytes, int* err, int num_sms, cudaStream_t st, int* nlaunch) {
  if (nlaunch) *nlaunch = 0;
  if (M <= 0) return cudaSuccess;
  int bn, splits, kps;
  gemm_plan(w, M, num_sms, &bn, &splits, &kps);
  const int KT = w.k / kBK;
  const size_t slice = (size_t)M * w.n * sizeof(float);
  if (splits > 1 && splits * slice > ws_bytes) {  // fewer splits that fit the workspace
    const int fit = (int)std::min<size_t>(splits, ws_bytes / std::max<size_t>(slice, 1));
    splits = std::max(1, fit);
    kps = (KT + splits - 1) / splits;
    splits = (KT + kps - 1) / kps;
    if (splits * slice > ws_bytes) splits = 1, kps = KT;
  }
  CUtensorMap map;
  if (make_act_map(&map, act, M, w.k, lda, bn) != 0) return cudaErrorInvalidValue;
  TileGrid tg{w.npad / kBM, (M + bn - 1) / bn, splits, kps, KT};
  if (nlaunch) *nlaunch = splits == 1 ? 1 : 2;
  if (splits == 1)
    return silu ? launch_epi<kEpiSilu>(bn, map, w, M, tg, num_sms, y, ldy, nullptr, err, st)
                : launch_epi<kEpiStore>(bn, map, w, M, tg, num_sms, y, ldy, nullptr, err, st);
  cudaError_t e = launch_epi<kEpiPartial>(bn, map, w, M, tg, num_sms, y, ldy, ws, err, st);
  if (e != cudaSuccess) return e;
  const int64_t total = silu ? (int64_t)M * (w.n / 2) : (int64_t)M * w.n;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4096);
  gemm_finish<<<blocks, 256, 0, st>>>(ws, splits, M, w.n, y, ldy, silu ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t repack_weight(const uint8_t* q, const __half* s, int n, int k, bool interleave, QWeight* out, cudaStream_t st) {
  out->n = n;
  out->k = k;
  out->npad = (n + kBM - 1) / kBM * kBM;
  out->interleaved = interleave;
  const size_t bytes = (size_t)(out->npad / kBM) * (k / kBK) * kTileBytes;
  cudaError_t e = cudaMalloc(&out->tiles, bytes);
  if (e != cudaSuccess) return e;
  out->bytes = bytes;
  const int64_t total = (int64_t)out->npad * (k / kBK);
  repack_q4<<<(int)std::min<int64_t>((total + 255) / 256, 8192), 256, 0, st>>>(q, s, n, k, out->npad, interleave ? 1 : 0,
                                                                               out->tiles);
  return cudaGetLastError();
}

}  // namespace sd
