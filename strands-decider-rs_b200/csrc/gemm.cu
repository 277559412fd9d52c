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
  static constexpr int kStages = BN >= 256 ? 4 : (BN >= 128 ? 6 : (BN >= 64 ? 7 : 8));
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr size_t kA = (size_t)kBM * kBK * 2;
  static constexpr size_t kB = (size_t)BN * kBK * 2;
  static constexpr size_t kOffB = kStages * kA;
  static constexpr size_t kOffRaw = kOffB + kStages * kB;
  static constexpr size_t kOffBar = kOffRaw + (size_t)kStages * kTileBytes;
  static constexpr size_t kBytes = kOffBar + (3 * kStages + 1) * 8 + 16;
  static constexpr size_t kSmem = kBytes + 1024;  // room to align the base to 1024 bytes
};

enum Epi { kEpiStore = 0, kEpiSilu = 1, kEpiAtomic = 2 };

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_q4_tc(const __grid_constant__ CUtensorMap act_map, const uint8_t* __restrict__ wt, int M, int N, int K,
               int kt_per_split, __half* __restrict__ y, int ldy, float* __restrict__ ws, int* err) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = base;
  uint8_t* sb = base + Cfg::kOffB;
  uint8_t* sraw = base + Cfg::kOffRaw;
  uint64_t* full_raw = reinterpret_cast<uint64_t*>(base + Cfg::kOffBar);
  uint64_t* full_a = full_raw + S;
  uint64_t* empty = full_a + S;
  uint64_t* acc_full = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.x, mt = blockIdx.y;
  const int KT = K / kBK;
  const int kt0 = blockIdx.z * kt_per_split;
  const int kt1 = min(KT, kt0 + kt_per_split);
  const int nk = max(0, kt1 - kt0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full_raw[s], 1);
      mbar_init(&full_a[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
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

  if (warp == 0) {
    if (lane == 0 && nk > 0) {
      prefetch_tmap(&act_map);
      const uint8_t* wtile = wt + (size_t)nt * KT * kTileBytes;
      for (int i = 0; i < nk; i++) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (i >= S && !mbar_wait(&empty[s], ph ^ 1, abort, err, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full_raw[s], (uint32_t)(Cfg::kB + kTileBytes));
        tma_load_2d(sb + s * Cfg::kB, &act_map, &full_raw[s], (kt0 + i) * kBK, mt * BN);
        bulk_load(sraw + s * kTileBytes, wtile + (size_t)(kt0 + i) * kTileBytes, kTileBytes, &full_raw[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nk > 0) {
      constexpr uint32_t idesc = idesc_f16(kBM, BN);
      for (int i = 0; i < nk; i++) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(&full_a[s], ph, abort, err, kErrTimeoutFull)) break;
        tc_fence_after();
        const uint64_t ad = sw128_desc(sa + s * Cfg::kA);
        const uint64_t bd = sw128_desc(sb + s * Cfg::kB);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; kk++)  // 16 f16 = 32 bytes per step: +2 in the address field
          tc_mma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0);
        tc_commit(&empty[s]);
      }
      tc_commit(acc_full);
    }
  } else {
    // Dequantization: thread r owns weight row r of the tile.
    const int r = threadIdx.x - 64;
    for (int i = 0; i < nk; i++) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      if (!mbar_wait(&full_raw[s], ph, abort, err, kErrTimeoutFull)) break;
      const uint8_t* raw = sraw + s * kTileBytes;
      const uint4 c0 = *reinterpret_cast<const uint4*>(raw + r * 32);
      const uint4 c1 = *reinterpret_cast<const uint4*>(raw + r * 32 + 16);
      const __half2* sc = reinterpret_cast<const __half2*>(raw + kTileCodes) + r;
      const __half2 scp = *sc;
      const __half2 s0 = __low2half2(scp), s1 = __high2half2(scp);
      const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      uint8_t* arow = sa + s * Cfg::kA + r * 128;
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const __half2 sc2 = c < 4 ? s0 : s1;
        uint4 o;
        o.x = h2_as_u32(dq_pair(w[c], 0, sc2));
        o.y = h2_as_u32(dq_pair(w[c], 1, sc2));
        o.z = h2_as_u32(dq_pair(w[c], 2, sc2));
        o.w = h2_as_u32(dq_pair(w[c], 3, sc2));
        *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) = o;
      }
      fence_proxy_async_smem();
      mbar_arrive(&full_a[s]);
    }
    // Epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31, i.e. weight rows of the tile.
    if (nk > 0 && mbar_wait(acc_full, 0, abort, err, kErrTimeoutAccum)) {
      tc_fence_after();
      const int q = warp & 3;
      const int n = nt * kBM + q * 32 + lane;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + c0, v);
        tc_wait_ld();
        const int mbase = mt * BN + c0;
        if (mbase >= M) break;
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const int m = mbase + j;
          const float acc = __uint_as_float(v[j]);
          if (EPI == kEpiStore) {
            if (m < M && n < N) y[(size_t)m * ldy + n] = __float2half_rn(acc);
          } else if (EPI == kEpiSilu) {
            // rows interleaved as (gate j, up j): even lanes hold gate, odd lanes up
            const float g = __half2float(__float2half_rn(acc));
            const float u = __shfl_xor_sync(0xffffffffu, g, 1);
            if ((lane & 1) == 0 && m < M && n < N) y[(size_t)m * ldy + (n >> 1)] = __float2half_rn(g / (1.0f + __expf(-g)) * u);
          } else {
            if (m < M && n < N) atomicAdd(ws + (size_t)m * N + n, acc);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// Split-K finish: f32 partial sums -> f16 (or SwiGLU of interleaved gate/up rows).
__global__ void gemm_finish(const float* __restrict__ ws, int M, int N, __half* __restrict__ y, int ldy, int silu) {
  const int64_t total = silu ? (int64_t)M * (N / 2) : (int64_t)M * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    if (!silu) {
      const int64_t m = i / N, n = i % N;
      y[m * ldy + n] = __float2half_rn(ws[i]);
    } else {
      const int64_t half = N / 2, m = i / half, j = i % half;
      const float g = __half2float(__float2half_rn(ws[m * N + 2 * j]));
      const float u = __half2float(__float2half_rn(ws[m * N + 2 * j + 1]));
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
static cudaError_t launch_bn(const CUtensorMap& map, const QWeight& w, int M, int splits, int kt_per_split, __half* y, int ldy,
                             float* ws, int* err, cudaStream_t st) {
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
  dim3 grid(w.npad / kBM, (M + BN - 1) / BN, splits);
  kern<<<grid, 192, Cfg::kSmem, st>>>(map, w.tiles, M, w.n, w.k, kt_per_split, y, ldy, ws, err);
  return cudaGetLastError();
}

template <int EPI>
static cudaError_t launch_epi(int bn, const CUtensorMap& map, const QWeight& w, int M, int splits, int kps, __half* y, int ldy,
                              float* ws, int* err, cudaStream_t st) {
  switch (bn) {
    case 32: return launch_bn<32, EPI>(map, w, M, splits, kps, y, ldy, ws, err, st);
    case 64: return launch_bn<64, EPI>(map, w, M, splits, kps, y, ldy, ws, err, st);
    case 128: return launch_bn<128, EPI>(map, w, M, splits, kps, y, ldy, ws, err, st);
    default: return launch_bn<256, EPI>(map, w, M, splits, kps, y, ldy, ws, err, st);
  }
}

void gemm_plan(const QWeight& w, int M, int num_sms, int* bn_out, int* splits_out, int* kps_out) {
  int bn = M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256));
  const int ntiles = w.npad / kBM;
  // Prefer 128-wide token tiles when 256-wide ones leave most SMs idle.
  if (bn == 256 && (int64_t)ntiles * ((M + 255) / 256) < num_sms) bn = 128;
  const int mtiles = (M + bn - 1) / bn;
  const int KT = w.k / kBK;
  int splits = 1;
  const int ctas = ntiles * mtiles;
  if (ctas < num_sms) {
    splits = (num_sms + ctas - 1) / ctas;
    splits = std::min(splits, std::max(1, KT / 4));  // at least 4 k-tiles per split
  }
  const int kps = (KT + splits - 1) / splits;
  splits = (KT + kps - 1) / kps;
  *bn_out = bn;
  *splits_out = splits;
  *kps_out = kps;
}

// y[M][ldy] = act[M][K] W^T (or SwiGLU of interleaved gate/up rows into y[M][N/2] when silu).
cudaError_t gemm_q4(const QWeight& w, const __half* act, int M, int lda, __half* y, int ldy, bool silu, float* ws,
                    size_t ws_bytes, int* err, int num_sms, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  int bn, splits, kps;
  gemm_plan(w, M, num_sms, &bn, &splits, &kps);
  if (splits > 1 && (size_t)M * w.n * sizeof(float) > ws_bytes) {
    splits = 1;
    kps = w.k / kBK;
  }
  CUtensorMap map;
  if (make_act_map(&map, act, M, w.k, lda, bn) != 0) return cudaErrorInvalidValue;
  if (splits == 1)
    return silu ? launch_epi<kEpiSilu>(bn, map, w, M, 1, kps, y, ldy, nullptr, err, st)
                : launch_epi<kEpiStore>(bn, map, w, M, 1, kps, y, ldy, nullptr, err, st);
  cudaError_t e = cudaMemsetAsync(ws, 0, (size_t)M * w.n * sizeof(float), st);
  if (e != cudaSuccess) return e;
  e = launch_epi<kEpiAtomic>(bn, map, w, M, splits, kps, y, ldy, ws, err, st);
  if (e != cudaSuccess) return e;
  const int64_t total = silu ? (int64_t)M * (w.n / 2) : (int64_t)M * w.n;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4096);
  gemm_finish<<<blocks, 256, 0, st>>>(ws, M, w.n, y, ldy, silu ? 1 : 0);
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
