// The gated delta rule (the reference's `Gdn` kernels, src/kernels.rs:257-302) as one fused chunked
// scan on the 5th-generation tensor cores.
//
// Per token and head (src/kernels.rs:282-297): q^ = q rsqrt(|q|^2 + 1e-6) / sqrt(DK),
// k^ = k rsqrt(|k|^2 + 1e-6), S <- gamma S, delta = beta (v - S^T k^), S += k^ delta^T, o = S^T q^.
// Chunks of C = 64 tokens from the entry state S (DK x DV, f32), with G_i = sum_{j<=i} g_j and
// Gamma_i = exp(G_i) (the WY form of the chunk, as gdn.cu states it):
//   A_ij = beta_i e^{G_i - G_j} k^_i.k^_j (j < i),  T = (I + A)^-1,  T1 = T diag(beta Gamma),  T2 = T diag(beta)
//   W = T1 K^,  U = T2 V,  delta = U - W S,  P_ij = e^{G_i - G_j} q^_i.k^_j (j <= i)
//   (k^ = rk k, q^ = rq q: the norms below)
//   O = Gamma Q^ S + P delta,   S' = Gamma_C S + K^T diag(e^{G_C - G_i}) delta
//
// One CTA walks one (sequence, head) over all 128 value columns. The state S is the f32 accumulator
// of its own update in tensor memory. The chunk's products are tcgen05 MMAs of M = 128 that stack two
// 64-row operands: [K; Q] K^T gives A and P at once, [Gamma Q^; -W] S gives Gamma Q^ S and -W S
// (accumulated onto [0; U], so that the second half is delta), and [P; *] delta adds P delta to the
// first half. The state-independent work of chunk c + 1 (row norms, A and P, the triangular
// inverse, T1 and T2) runs beside the state chain of chunk c:
//   warps 0-3   the chain: O rows to global memory, S out of tensor memory (its f16 copy, the operand
//               of the next chunk, and Gamma_C S back), -W out of tensor memory, delta (f16, and
//               decayed as Ds); one thread issues U = [0; T2] V and the chain's MMAs ([Gamma Q^; -W] S,
//               K^T Ds, P delta) and the v rows' TMA, one the k and q rows' TMA (into the chunk's
//               tile), two chunks ahead at most;
//   warps 4-11  the chunk preparation: the norms of q and k, the gates and G, A and P from [K; Q] K^T, the
//               inverse (f32; 8 x 8 diagonal blocks by substitution, then doubled blocks, the larger
//               products on tf32 mma.sync), T1 and T2 (f16); their first thread issues [K; Q] K^T and
//               W = [T1; *] K, after which the chunk passes to the chain.
// Each group keeps its warps on the same path through its named barrier whatever happens (a wait
// that gives up marks the CTA aborted and the group skips the work that follows, not the barriers).
// The tile keeps k and q as loaded (f16): their norms, rk_i = rsqrt(|k_i|^2 + 1e-6) and
// rq_i = rsqrt(|q_i|^2 + 1e-6) / sqrt(DK), scale the f32 products instead (A and P by rows and columns,
// T1 by columns, Ds by rows, Gamma q^ = Gamma_i rq_i q_i), so no rounded q^ or k^ is formed. Rounded
// to f16: T1, T2, W, P, Gamma q^, delta, Ds and the state operand; f32 accumulation, U and the state.
//
// Every wait is bounded (2 s, common.cuh): a wait that runs out records an error code and the CTA
// winds down (each MMA issuer waits for its own MMAs, the TMA thread for its copies) without hanging.
#include <mutex>

#include "common.cuh"
#include "sd_internal.h"

namespace sd {

namespace {
constexpr int CH = 64, DK = 128;
constexpr int kThreads = 384;
constexpr int kBox = 192 * 128;                       // one 64-column half of a chunk tile: K^ rows 0-63, Q^ 64-127, W 128-191
constexpr int kTile = 2 * kBox;                       // 48 KB
constexpr int kOffKQW = 0;                            // [2] chunk tiles
constexpr int kOffV = kOffKQW + 2 * kTile;            // V: 64 tokens x 128 values, two 8 KB halves
constexpr int kOffS16 = kOffV + 16384;                // S (f16): 128 keys x 128 values, two 16 KB halves
constexpr int kOffT1 = kOffS16 + 32768;               // 8 KB tiles, in this order: T1 | P1 | P0 | Z | T2
constexpr int kOffP1 = kOffT1 + 8192;
constexpr int kOffP0 = kOffP1 + 8192;
constexpr int kOffZ = kOffP0 + 8192;
constexpr int kOffT2 = kOffZ + 8192;
// row stride (floats) of the f32 64 x 64 tiles: 4 mod 32 banks, so the tf32 MMA fragments' loads (rows g,
// columns t of an 8 x 4 lane grid) hit 32 different banks, and a row per lane stores 16-byte vectors
// at the minimum of four wavefronts
constexpr int LA = CH + 4;
constexpr int kOffA = kOffT2 + 8192;                  // A (f32), replaced in place by T = (I + A)^-1
constexpr int kOffY = kOffA + CH * LA * 4;            // 32 x 40 floats of the inverse's scratch
constexpr int kOffSmall = kOffY + 32 * 40 * 4;        // beta[2][64], G[2][64], g[64], decay tables E[64], Gam[64], F[4][64],
                                                      // row norms N[2][128]
constexpr int kOffBar = kOffSmall + 15 * CH * 4;
enum {
  B_KQ_FULL = 0,     // [2] the chunk's k and q rows landed (TMA bytes)
  B_V_FULL = 2,      // [2] the chunk's v rows landed
  B_U_DONE = 4,      // [2] U = [0; T2] V completed (T1 and T2 free; W read out before it)
  B_DAP_FULL = 6,    // [2] [K; Q] K^T in tensor memory
  B_W_FULL = 8,      // [2] W in tensor memory
  B_WQ_READY = 10,   // [2] Gamma Q^, P, T1 and T2 written (shared memory) and W issued
  B_G_READY = 12,    // [2] the chunk's G written
  B_X_FULL = 14,     // [2] [Gamma Q^; -W] S accumulated
  B_S_FULL = 16,     // [2] the state update completed
  B_O_FULL = 18,     // [2] P delta accumulated (O complete): every MMA of the chunk has completed
  B_O_READ = 20,     // [2] O read out of tensor memory and stored, its staging (P) read (2 arrivals)
  B_END_PREP = 22,   // every MMA of the preparation completed (teardown)
  B_END_CHAIN = 23,  // every MMA of the chain completed (teardown)
  kBars = 24
};
constexpr int kSmem = kOffBar + kBars * 8 + 16 + 1024;
static_assert(kSmem <= 232448, "shared memory");
constexpr uint32_t kColS = 0, kColX = 128, kColDAP = 384, kTmemCols = 512;
constexpr uint32_t kIdS = idesc_f16(128, 128) | (1u << 15) | (1u << 16);  // both operands MN-major
constexpr uint32_t kIdB = idesc_f16_bmn(128, 128);                        // B MN-major
constexpr uint32_t kIdAP = idesc_f16(128, 64);                            // both K-major
constexpr int kPrepBar = 1;                                               // named barrier of the preparation warps
constexpr int kChainBar = 2;                                              // named barrier of the chain warps

__device__ int g_gdn_tc_err;  // error slot of calls without one

// Byte offset of 16-byte piece `c` of row `r` in a tile stored with the 128-byte swizzle (rows of
// 128 bytes; the tile starts on a 1024-byte boundary).
SD_DEV uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

SD_DEV void prep_sync() { asm volatile("bar.sync %0, 256;" ::"n"(kPrepBar) : "memory"); }
SD_DEV void chain_sync() { asm volatile("bar.sync %0, 128;" ::"n"(kChainBar) : "memory"); }

// e^x as one ex2.approx.ftz (results below 2^-126 flush to zero). __expf without -ftz becomes a
// longer sequence that keeps denormal results, and the preparation takes thousands per chunk.
SD_DEV float fexp(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
  return y;
}

SD_DEV uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// A tf32 operand: the f32 bits as they are (the tensor cores read the top 19 bits, so this truncates
// the mantissa to 10 bits; T is rounded to f16 right after its products, which is coarser).
SD_DEV uint32_t tf32(float x) { return __float_as_uint(x); }
SD_DEV void mma1688_tf32(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 16 x 8 tile of a product of f32 matrices in shared memory on the tensor cores (tf32 operands: the
// top 19 bits of each f32, so the mantissa is truncated to 10 bits; f32 accumulation):
// acc += L[r0 .. r0 + 16)[k0 .. k1) R[k0 .. k1)[c0 .. c0 + 8), k1 - k0 a multiple of 8.
SD_DEV void mm_tile(float (&acc)[4], const float* __restrict__ L, int ldl, const float* __restrict__ R, int ldr, int r0, int c0,
                    int k0, int k1, int g, int tq) {
  for (int k = k0; k < k1; k += 8) {
    const float* lp = L + (r0 + g) * ldl + k;
    const float* rp = R + (k + tq) * ldr + c0 + g;
    mma1688_tf32(acc, tf32(lp[tq]), tf32(lp[8 * ldl + tq]), tf32(lp[tq + 4]), tf32(lp[8 * ldl + tq + 4]), tf32(rp[0]),
                 tf32(rp[4 * ldr]));
  }
}
SD_DEV void st_tile(float* __restrict__ D, int ldd, int r0, int c0, const float (&acc)[4], float sign, int g, int tq) {
  D[(r0 + g) * ldd + c0 + 2 * tq] = sign * acc[0];
  D[(r0 + g) * ldd + c0 + 2 * tq + 1] = sign * acc[1];
  D[(r0 + g + 8) * ldd + c0 + 2 * tq] = sign * acc[2];
  D[(r0 + g + 8) * ldd + c0 + 2 * tq + 1] = sign * acc[3];
}

// X = (I + A)^-1 for the strictly lower triangular 64 x 64 A (rows LA floats apart), in place, by the
// eight preparation warps (pw = 0..7, pt = 0..255), doubling the inverted blocks: the eight 8 x 8
// diagonal blocks by forward substitution (warp pw, lane = column), then the lower-left block of each
// 2s x 2s diagonal block from its two s x s halves, X_10 = -X_11 (A_10 X_00), for s = 8 (four blocks,
// on the CUDA cores), 16 (two blocks) and 32 (one block), the last two on the tensor cores. Each A_10
// is read (into Y) before X_10 replaces it, and no level reads an A block an earlier level replaced.
// The array must hold zeros above the diagonal (the products read whole s x s blocks; A's rows are
// written whole, zeros included, and no level writes there). `y`: 32 x 40 floats of scratch (row strides
// of 24 and 40: 8 mod 32 banks for the B fragments' loads).
SD_DEV void tri_inverse(float* a, float* y, int pw, int pt, int lane) {
  float* x = a;
  const int o = pw * 8, c = lane;
  float xc[8];
  if (lane < 8) {
#pragma unroll
    for (int r = 0; r < 8; r++) {  // branch-free: xc[j] is zero above the diagonal (j < c)
      float v = r == c ? 1.0f : 0.0f;
#pragma unroll
      for (int j = 0; j < r; j++) v -= a[(o + r) * LA + o + j] * xc[j];
      xc[r] = r >= c ? v : 0.0f;
    }
  }
  __syncwarp();  // the block's A read before its T is written over it
  if (lane < 8) {
#pragma unroll
    for (int r = 0; r < 8; r++) x[(o + r) * LA + o + c] = xc[r];
  }
  prep_sync();
  {  // s = 8: thread pt takes element (i, j) of block b = pt / 64 (rows 16 b + 8 .., columns 16 b ..)
    const int b = pt >> 6, i = (pt >> 3) & 7, jj = pt & 7, o = 16 * b;
    float t = 0.0f;
#pragma unroll
    for (int m = 0; m < 8; m++) t += a[(o + 8 + i) * LA + o + m] * x[(o + m) * LA + o + jj];
    y[b * 64 + i * 8 + jj] = t;
    prep_sync();
    float z = 0.0f;
#pragma unroll
    for (int m = 0; m < 8; m++) z += x[(o + 8 + i) * LA + o + 8 + m] * y[b * 64 + m * 8 + jj];
    x[(o + 8 + i) * LA + o + jj] = -z;
  }
  prep_sync();
  const int g = lane >> 2, tq = lane & 3;
  {  // s = 16: warps 0-3, block b = pw / 2 (rows 32 b + 16 .., columns 32 b ..), 8 columns each
    const int b = (pw >> 1) & 1, c0 = 8 * (pw & 1), o = 32 * b;
    float* yb = y + b * 16 * 24;
    if (pw < 4) {
      float acc[4] = {};
      mm_tile(acc, a + (o + 16) * LA + o, LA, x + o * LA + o, LA, 0, c0, 0, 16, g, tq);
      st_tile(yb, 24, 0, c0, acc, 1.0f, g, tq);
    }
    prep_sync();
    if (pw < 4) {
      float acc[4] = {};
      mm_tile(acc, x + (o + 16) * LA + o + 16, LA, yb, 24, 0, c0, 0, 16, g, tq);
      st_tile(x + (o + 16) * LA + o, LA, 0, c0, acc, -1.0f, g, tq);
    }
  }
  prep_sync();
  {  // s = 32: eight warps, a 16 x 8 tile each of the 32 x 32 block (rows 32 .., columns 0 ..)
    const int r0 = 16 * (pw & 1), c0 = 8 * (pw >> 1);
    float acc[4] = {};
    mm_tile(acc, a + 32 * LA, LA, x, LA, r0, c0, 0, 32, g, tq);
    st_tile(y, 40, r0, c0, acc, 1.0f, g, tq);
    prep_sync();
    float acc2[4] = {};
    mm_tile(acc2, x + 32 * LA + 32, LA, y, 40, r0, c0, 0, 32, g, tq);
    st_tile(x + 32 * LA, LA, r0, c0, acc2, -1.0f, g, tq);
  }
  prep_sync();
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    gdn_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap omap, const GdnTcArgs a) {
  grid_dep_wait();  // launched as a programmatic dependent (launch_dependent): inputs ready from here
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = smem_align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sbeta = reinterpret_cast<float*>(base + kOffSmall);  // [2][64]
  float* sG = sbeta + 2 * CH;                                  // [2][64]
  float* sg = sG + 2 * CH;                                     // [64]
  // the chunk's decays, made once per chunk so that the A and P rows need few exponentials: with
  // block b = i / 16 of row i and M_b = G_{16 b}, e^{G_i - G_j} = E_i F_{b,j} for j < 16 b, where
  // E_i = e^{G_i - M_b} and F_{b,j} = e^{M_b - G_j} are both at most 1 (G never increases), so neither
  // factor can overflow; pairs within one block take their own exponential. Gam_j = e^{G_j}.
  float* sE = sg + CH;                                         // [64]
  float* sGam = sE + CH;                                       // [64]
  float* sF = sGam + CH;                                       // [4][64]
  // rsqrt(|k_i|^2 + 1e-6) (rows 0-63) and rsqrt(|q_i|^2 + 1e-6) / sqrt(DK) (rows 64-127) of chunk c
  // (sN[c & 1]): the tile keeps the raw k and q, and the products take these as row and column scales
  float* sN = sF + 4 * CH;                                     // [2][128]
  int* err = a.err ? a.err : &g_gdn_tc_err;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.h;

  // this CTA's walk: sequence b (its tokens tok0 .. tok0 + L - 1 of the gates and outputs; of the
  // q/k/v maps rows y0 .. in slab z), head hd
  const int hd = blockIdx.x % H;
  int b, L, z;
  long long tok0, y0;
  const float* sin;
  float* sout;
  const long long hoff = (long long)hd * DK * DK;
  if (a.seq_off) {
    b = a.order ? a.order[blockIdx.x / H] : blockIdx.x / H;
    tok0 = a.seq_off[b];
    L = a.seq_len[b];
    z = 0;
    y0 = tok0;
    sin = a.s_in && a.s_in[b] ? a.s_in[b] + hoff : nullptr;
    sout = a.s_out && a.s_out[b] ? a.s_out[b] + hoff : nullptr;
  } else {
    b = blockIdx.x / H;
    L = a.l;
    tok0 = (long long)b * a.l;
    z = b;
    y0 = 0;
    const long long sb = (long long)H * DK * DK;
    sin = a.load_state ? a.state + b * sb + hoff : nullptr;
    sout = a.store_state ? a.state + b * sb + hoff : nullptr;
  }
  const int nch = (L + CH - 1) / CH;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kBars; i++) mbar_init(&bar[i], i >= B_O_READ && i < B_O_READ + 2 ? 2 : 1);
    *abort = 0;
    fence_mbar_init();
  }
  // the zero tile (rows 0-63 of U's [0; T2] operand)
  for (int i = threadIdx.x; i < 8192 / 16; i += kThreads) reinterpret_cast<uint4*>(base + kOffZ)[i] = make_uint4(0, 0, 0, 0);
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (nch == 0) {
    // nothing to walk: the final state is the initial one
  } else if (warp < 4) {
    // ---------------------------------------------------------------- the chain (and the copies)
    const int q4 = warp;                           // TMEM lanes 32 q4 .. + 31
    const int r = q4 * 32 + lane;                  // S: key row r; D_X: row r
    const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
    const int x = hd * DK;
    // TMA of chunk c's k and q rows into its tile, and of its v rows
    auto load_kq = [&](int c) {
      const int s = c & 1, y = (int)(y0 + (long long)c * CH);
      uint8_t* t = base + kOffKQW + s * kTile;
      mbar_arrive_expect_tx(&bar[B_KQ_FULL + s], 4 * 8192);
      for (int hb = 0; hb < 2; hb++) {
        tma_load_3d(t + hb * kBox, &kmap, &bar[B_KQ_FULL + s], x + hb * 64, y, z);
        tma_load_3d(t + hb * kBox + 64 * 128, &qmap, &bar[B_KQ_FULL + s], x + hb * 64, y, z);
      }
    };
    auto load_v = [&](int c) {
      const int s = c & 1, y = (int)(y0 + (long long)c * CH);
      mbar_arrive_expect_tx(&bar[B_V_FULL + s], 2 * 8192);
      for (int hb = 0; hb < 2; hb++) tma_load_3d(base + kOffV + hb * 8192, &vmap, &bar[B_V_FULL + s], x + hb * 64, y, z);
    };
    int nkq = 0, nv = 0;  // copies issued (warp 0 lane 0: k/q; warp 2 lane 0: v)
    if (warp == 0 && lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      prefetch_tmap(&omap);
      for (; nkq < min(2, nch); nkq++) load_kq(nkq);
    }
    if (warp == 2 && lane == 0) load_v(nv++);
    // the entry state into tensor memory (zeros without one)
    for (int cb = 0; cb < 4; cb++) {
      uint32_t v[32];
      if (sin) {
        const float4* src = reinterpret_cast<const float4*>(sin + (size_t)r * DK + cb * 32);
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float4 f = src[i];
          v[4 * i] = __float_as_uint(f.x), v[4 * i + 1] = __float_as_uint(f.y);
          v[4 * i + 2] = __float_as_uint(f.z), v[4 * i + 3] = __float_as_uint(f.w);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = 0u;
      }
      tmem_st32(tmem + lanes + kColS + cb * 32, v);
    }
    tc_wait_st();
    bool ok = true;
    // O rows (D_X rows 0-63, warps 0 and 1) of chunk c to global memory, then D_X[c & 1] is released;
    // the MMAs of chunk c have all completed, so its tile takes chunk c + 2's k and q rows. A warp whose
    // 32 rows all lie in the sequence stores them as four 32 x 32 blocks through shared memory (chunk c's
    // P tile, 4 KB per warp: free once P delta of chunk c has completed, until the preparation of chunk
    // c + 2 writes P there, which waits for this read-out) with the TMA, in whole 128-byte lines:
    // lane-per-row stores from the registers would write 32 rows' 16-byte pieces per instruction and hold
    // up the shared-memory traffic of the preparation warps beside them. (Other MMAs read the tile only as
    // the spare rows 64-127 of an M = 128 operand, whose products are not used.) The ragged rows of a
    // last chunk are stored directly.
    auto read_o = [&](int c) {
      const int s = c & 1;
      if (ok) ok = mbar_wait_warp<false>(&bar[B_O_FULL + s], (c >> 1) & 1, abort, err, kErrTimeoutAccum);
      if (ok && warp == 0 && lane == 0 && c + 2 < nch) load_kq(nkq++);
      if (ok && q4 < 2) {
        tc_fence_after();
        const int n = min(CH, L - c * CH);
        const bool whole = n >= 32 * (q4 + 1);
        uint8_t* stage = base + (s ? kOffP1 : kOffP0) + q4 * 4096;
        // tcgen05.ld and wait::ld are warp-collective (.sync.aligned): every lane of the warp executes
        // the same loads, and only the stores are limited to the chunk's rows
        float* dst = a.o + (size_t)(tok0 + c * CH + r) * H * DK + hd * DK;
        for (int cb = 0; cb < 4; cb++) {
          uint32_t v[32];
          tmem_ld32(tmem + lanes + kColX + s * 128 + cb * 32, v);
          tc_wait_ld();
          if (whole) {
            if (cb > 0) {  // the previous block's store has read the staging
              if (lane == 0) bulk_wait_read();
              __syncwarp();
            }
#pragma unroll
            for (int i = 0; i < 8; i++)
              *reinterpret_cast<uint4*>(stage + lane * 128 + ((i ^ (lane & 7)) << 4)) =
                  make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&omap, stage, hd * DK + cb * 32, (int)(tok0 + c * CH + q4 * 32));
              bulk_commit();
            }
          } else if (r < n) {
            float4* d4 = reinterpret_cast<float4*>(dst + cb * 32);
#pragma unroll
            for (int i = 0; i < 8; i++)
              d4[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), __uint_as_float(v[4 * i + 2]),
                                  __uint_as_float(v[4 * i + 3]));
          }
        }
        if (whole && lane == 0) bulk_wait_read();
      }
      tc_fence_before();
      __syncwarp();
      // warps 0 and 1 only: warps 2 and 3 read their rows (delta) before the chunk's last MMAs were
      // issued, and warp 2 reaches this point only after the next chunk's preparation, which waits here
      if (lane == 0 && q4 < 2) mbar_arrive(&bar[B_O_READ + s]);
    };
    for (int c = 0; c < nch; c++) {
      const int s = c & 1;
      const uint32_t ph = (c >> 1) & 1;
      uint8_t* t = base + kOffKQW + s * kTile;
      const uint32_t dx = tmem + kColX + s * 128;
      // (0) O of the previous chunk first (the next chunk's preparation waits for it before it writes T1)
      if (c >= 1) read_o(c - 1);
      // (1) the entry state S_{c-1}: its f16 copy (the operand of [Gamma Q^; -W] S), Gamma_C S back
      if (ok && c >= 1) ok = mbar_wait_warp<false>(&bar[B_S_FULL + (s ^ 1)], ((c - 1) >> 1) & 1, abort, err, kErrTimeoutAccum);
      if (ok) ok = mbar_wait_warp<false>(&bar[B_G_READY + s], ph, abort, err, kErrTimeoutFull);
      if (ok) {
        tc_fence_after();
        const float gc = fexp(sG[s * CH + CH - 1]);
        for (int cb = 0; cb < 4; cb++) {
          uint32_t v[32];
          tmem_ld32(tmem + lanes + kColS + cb * 32, v);
          tc_wait_ld();
          uint8_t* dst = base + kOffS16 + (cb >> 1) * 16384;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            uint4 u;
            u.x = pack_h2(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1]));
            u.y = pack_h2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
            u.z = pack_h2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
            u.w = pack_h2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
            *reinterpret_cast<uint4*>(dst + swz(r, (cb & 1) * 4 + j)) = u;
          }
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = __float_as_uint(__uint_as_float(v[i]) * gc);
          tmem_st32(tmem + lanes + kColS + cb * 32, v);
        }
        tc_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      if (!__all_sync(0xffffffffu, ok)) *abort = 1;
      chain_sync();
      ok = ok && !*abort;
      // (2) -W (D_X rows 0-63, warps 0 and 1) over rows 128-191 of the tile, once W has completed; the
      // preparation has gone on to the next chunk
      if (ok && q4 < 2) {
        ok = mbar_wait_warp<false>(&bar[B_W_FULL + s], ph, abort, err, kErrTimeoutAccum);
        if (ok) {
          tc_fence_after();
          for (int cb = 0; cb < 4; cb++) {
            uint32_t v[32];
            tmem_ld32(dx + lanes + cb * 32, v);
            tc_wait_ld();
            uint8_t* box = t + (cb >> 1) * kBox;
#pragma unroll
            for (int j = 0; j < 4; j++)
              *reinterpret_cast<uint4*>(box + swz(128 + r, (cb & 1) * 4 + j)) =
                  make_uint4(pack_h2(-__uint_as_float(v[8 * j]), -__uint_as_float(v[8 * j + 1])),
                             pack_h2(-__uint_as_float(v[8 * j + 2]), -__uint_as_float(v[8 * j + 3])),
                             pack_h2(-__uint_as_float(v[8 * j + 4]), -__uint_as_float(v[8 * j + 5])),
                             pack_h2(-__uint_as_float(v[8 * j + 6]), -__uint_as_float(v[8 * j + 7])));
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      if (!__all_sync(0xffffffffu, ok)) *abort = 1;
      chain_sync();
      ok = ok && !*abort;
      if (warp == 2) {  // U = [0; T2] V into D_X[s] (rows 0-63 zero), then [Gamma Q^; -W] S onto it (rows
                        // 0-63 Gamma Q^ S, rows 64-127 delta)
        if (ok) ok = mbar_wait_warp<false>(&bar[B_WQ_READY + s], ph, abort, err, kErrTimeoutFull);
        if (ok) ok = mbar_wait_warp<false>(&bar[B_V_FULL + s], ph, abort, err, kErrTimeoutFull);
        if (ok && lane == 0) {
          tc_fence_after();
          {
            const uint64_t ad = sw128_desc(base + kOffZ), bd = sw128_mn_desc(base + kOffV, 8192);
#pragma unroll
            for (int ks = 0; ks < 4; ks++) tc_mma_f16(dx, ad + (uint64_t)(2 * ks), bd + (uint64_t)(128 * ks), kIdB, ks > 0);
          }
          tc_commit(&bar[B_U_DONE + s]);
          const uint64_t ad = sw128_desc(t + 64 * 128), bd = sw128_mn_desc(base + kOffS16, 16384);
#pragma unroll
          for (int ks = 0; ks < 8; ks++)
            tc_mma_f16(dx, ad + (uint64_t)((ks >> 2) * (kBox >> 4) + 2 * (ks & 3)), bd + (uint64_t)(128 * ks), kIdB, 1);
          tc_commit(&bar[B_X_FULL + s]);
        }
      }
      // (3) delta = D_X rows 64-127 (warps 2 and 3): delta (f16, over Gamma Q^) and Ds = delta e^{G_C - G_i}
      // (over -W)
      if (ok) ok = mbar_wait_warp<false>(&bar[B_X_FULL + s], ph, abort, err, kErrTimeoutAccum);
      if (ok && warp == 2 && lane == 0 && c + 1 < nch) load_v(nv++);  // the v buffer is free: U has completed
      if (ok && q4 >= 2) {
        tc_fence_after();
        const int i = r - 64;
        const float sc = fexp(sG[s * CH + CH - 1] - sG[s * CH + i]) * sN[s * 128 + i];  // K^T Ds = K^T (rk Ds)
        for (int cb = 0; cb < 4; cb++) {
          uint32_t v[32];
          tmem_ld32(tmem + lanes + kColX + s * 128 + cb * 32, v);
          tc_wait_ld();
          uint8_t* box = t + (cb >> 1) * kBox;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            uint4 u, w;
            u.x = pack_h2(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1]));
            u.y = pack_h2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
            u.z = pack_h2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
            u.w = pack_h2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
            w.x = pack_h2(__uint_as_float(v[8 * j]) * sc, __uint_as_float(v[8 * j + 1]) * sc);
            w.y = pack_h2(__uint_as_float(v[8 * j + 2]) * sc, __uint_as_float(v[8 * j + 3]) * sc);
            w.z = pack_h2(__uint_as_float(v[8 * j + 4]) * sc, __uint_as_float(v[8 * j + 5]) * sc);
            w.w = pack_h2(__uint_as_float(v[8 * j + 6]) * sc, __uint_as_float(v[8 * j + 7]) * sc);
            *reinterpret_cast<uint4*>(box + swz(64 + i, (cb & 1) * 4 + j)) = u;
            *reinterpret_cast<uint4*>(box + swz(128 + i, (cb & 1) * 4 + j)) = w;
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      if (!__all_sync(0xffffffffu, ok)) *abort = 1;
      chain_sync();
      ok = ok && !*abort;
      if (warp == 2 && lane == 0 && ok) {  // S += K^T Ds, then O += [P; *] delta
        tc_fence_after();
        {
          const uint64_t ad = sw128_mn_desc(t, kBox), bd = sw128_mn_desc(t + 128 * 128, kBox);
#pragma unroll
          for (int ks = 0; ks < 4; ks++) tc_mma_f16(tmem + kColS, ad + (uint64_t)(128 * ks), bd + (uint64_t)(128 * ks), kIdS, 1);
        }
        tc_commit(&bar[B_S_FULL + s]);
        {  // the operand's rows 64-127 are whatever follows P
          const uint64_t ad = sw128_desc(base + (s ? kOffP1 : kOffP0)), bd = sw128_mn_desc(t + 64 * 128, kBox);
#pragma unroll
          for (int ks = 0; ks < 4; ks++) tc_mma_f16(dx, ad + (uint64_t)(2 * ks), bd + (uint64_t)(128 * ks), kIdB, 1);
        }
        tc_commit(&bar[B_O_FULL + s]);
      }
    }
    read_o(nch - 1);
    if (q4 < 2 && lane == 0) bulk_wait_all();  // the output stores have completed
    // the final state
    if (ok && sout) {
      const int c = nch - 1;
      if ((ok = mbar_wait_warp<false>(&bar[B_S_FULL + (c & 1)], (c >> 1) & 1, abort, err, kErrTimeoutAccum))) {
        tc_fence_after();
        for (int cb = 0; cb < 4; cb++) {
          uint32_t v[32];
          tmem_ld32(tmem + lanes + kColS + cb * 32, v);
          tc_wait_ld();
          float4* d4 = reinterpret_cast<float4*>(sout + (size_t)r * DK + cb * 32);
#pragma unroll
          for (int i = 0; i < 8; i++)
            d4[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), __uint_as_float(v[4 * i + 2]),
                                __uint_as_float(v[4 * i + 3]));
        }
      }
    }
    // teardown: every MMA this group issued has completed, and no copy lands after the CTA has left
    if (warp == 2 && lane == 0) {
      tc_commit(&bar[B_END_CHAIN]);
      mbar_drain(&bar[B_END_CHAIN], 0);
      if (nv > 0) mbar_drain(&bar[B_V_FULL + ((nv - 1) & 1)], ((nv - 1) >> 1) & 1);
    }
    if (warp == 0 && lane == 0)
      for (int c = max(0, nkq - 2); c < nkq; c++) mbar_drain(&bar[B_KQ_FULL + (c & 1)], (c >> 1) & 1);
  } else {
    // ---------------------------------------------------------------- the chunk preparation
    const int pw = warp - 4;                  // 0..7
    const int pt = threadIdx.x - 4 * 32;      // 0..255
    const int q4 = warp & 3;                  // TMEM lanes 32 q4 .. + 31: K rows for q4 0, 1; Q rows for 2, 3
    const int colh = pw >> 2;                 // the half of the columns this warp takes of its lanes' rows
    const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
    float* sa = reinterpret_cast<float*>(base + kOffA);
    float* sy = reinterpret_cast<float*>(base + kOffY);
    const float qscale = rsqrtf((float)DK);
    bool ok = true;
    // the gates of chunk c, loaded one chunk ahead: g of positions 2 lane and 2 lane + 1 in every warp
    // (each warp scans G itself), beta by threads 0-63
    auto gates = [&](int c, float& g0, float& g1, float& bt) {
      g0 = g1 = bt = 0.0f;
      if (c >= nch) return;
      const long long t = tok0 + (long long)c * CH;
      const int n = min(CH, L - c * CH);
      if (2 * lane < n) g0 = a.g[(t + 2 * lane) * H + hd];
      if (2 * lane + 1 < n) g1 = a.g[(t + 2 * lane + 1) * H + hd];
      if (pt < n && pt < 64) bt = a.beta[(t + pt) * H + hd];
    };
    float gn0, gn1, bn;
    gates(0, gn0, gn1, bn);
    for (int c = 0; c < nch; c++) {
      const int s = c & 1;
      const uint32_t ph = (c >> 1) & 1;
      uint8_t* t = base + kOffKQW + s * kTile;
      const uint32_t dx = tmem + kColX + s * 128;
      const float g0 = gn0, g1 = gn1, bc = bn;
      gates(c + 1, gn0, gn1, bn);
      // (1) the chunk's raw k and q rows: [K; Q] K^T at once (rows 0-63 K K^T, rows 64-127 Q K^T); the
      // gates, G and the decay tables, and the rows' norms beside it (G[s], beta[s] and N[s] are free:
      // the chain's last use of them, chunk c - 2, came before the chunk c - 1 read-out that the
      // preparation of chunk c - 1 waited for)
      if (ok) ok = mbar_wait_warp<false>(&bar[B_KQ_FULL + s], ph, abort, err, kErrTimeoutFull);
      if (pt == 0 && ok) {
        tc_fence_after();
        const uint64_t ad = sw128_desc(t);
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          const uint64_t o = (uint64_t)((ks >> 2) * (kBox >> 4) + 2 * (ks & 3));
          tc_mma_f16(tmem + kColDAP, ad + o, ad + o, kIdAP, ks > 0);
        }
        tc_commit(&bar[B_DAP_FULL + s]);
      }
      if (pt < 64) sbeta[s * CH + pt] = bc;
      {  // G = inclusive prefix sums of g (every warp: lane l holds G_{2l}, G_{2l+1}), then the decays
        float sum = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float u = __shfl_up_sync(0xffffffffu, sum, o);
          if (lane >= o) sum += u;
        }
        const float G0 = sum - g1, G1 = sum;
        if (pw == 0) {
          sG[s * CH + 2 * lane] = G0;
          sG[s * CH + 2 * lane + 1] = G1;
        }
        auto g_at = [&](int j) {
          const float u0 = __shfl_sync(0xffffffffu, G0, j >> 1), u1 = __shfl_sync(0xffffffffu, G1, j >> 1);
          return (j & 1) ? u1 : u0;
        };
        const int b4 = pt >> 6, j = pt & 63;
        const float gj = g_at(j), gm = g_at(16 * b4), gb = g_at(j & ~15);
        sF[pt] = j < 16 * b4 ? fexp(gm - gj) : 0.0f;
        if (pt < 64) sE[pt] = fexp(gj - gb);
        else if (pt < 128) sGam[j] = fexp(gj);
      }
      // (2) the row norms: thread pt takes one 64-column half (pt & 1) of row pt >> 1 (rows 0-63 k,
      // 64-127 q); the two halves' sums of squares meet through one shuffle
      if (ok) {
        const int row = pt >> 1, hb = pt & 1;
        const uint8_t* rp = t + hb * kBox;
        uint4 raw[8];
#pragma unroll
        for (int j = 0; j < 8; j++) raw[j] = *reinterpret_cast<const uint4*>(rp + swz(row, j));
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const uint32_t* w = reinterpret_cast<const uint32_t*>(&raw[j]);
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
            ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
          }
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        if (hb == 0) sN[s * 128 + row] = row < 64 ? rsqrtf(ss + 1e-6f) : rsqrtf(ss + 1e-6f) * qscale;
      }
      prep_sync();
      if (pt == 0) mbar_arrive(&bar[B_G_READY + s]);
      // (3) A (K rows) and P (Q rows) from the products, each warp 32 of the 64 columns of its lanes'
      // rows; Gamma Q^ over Q^ (each warp one 64-column half)
      if (ok) ok = mbar_wait_warp<false>(&bar[B_DAP_FULL + s], ph, abort, err, kErrTimeoutAccum);
      if (ok && q4 >= 2 && c >= 2)  // P[s] is free once the chain has stored chunk c - 2's O through it
        ok = mbar_wait_warp<false>(&bar[B_O_READ + s], ((c >> 1) - 1) & 1, abort, err, kErrTimeoutEmpty);
      if (ok) {
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(tmem + lanes + kColDAP + 32 * colh, v);
        tc_wait_ld();
        const float* G = sG + s * CH;
        const int j0 = 32 * colh;
        // G of this warp's 32 columns into registers first: the stores below go to shared memory too,
        // and loads interleaved with them could not be moved ahead of them
        float gj[32];
#pragma unroll
        for (int j4 = 0; j4 < 8; j4++) {
          const float4 f = *reinterpret_cast<const float4*>(G + j0 + 4 * j4);
          gj[4 * j4] = f.x, gj[4 * j4 + 1] = f.y, gj[4 * j4 + 2] = f.z, gj[4 * j4 + 3] = f.w;
        }
        // the decays of row i's 32 columns j (two 16-column blocks): E_i F_{b,j} in the blocks before
        // row i's, e^{G_i - G_j} in its own (the only exponentials), zero after it
        const int i = (q4 & 1) * 32 + lane, bi_ = i >> 4;
        const float gi = G[i], ei = sE[i];
        float dec[32];
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          const int bj = (j0 >> 4) + hf;
          if (bj < bi_) {
#pragma unroll
            for (int e = 0; e < 16; e++) dec[16 * hf + e] = ei * sF[bi_ * CH + 16 * bj + e];
          } else if (bj == bi_) {
#pragma unroll
            for (int e = 0; e < 16; e++) dec[16 * hf + e] = 16 * bj + e <= i ? fexp(gi - gj[16 * hf + e]) : 0.0f;
          } else {
#pragma unroll
            for (int e = 0; e < 16; e++) dec[16 * hf + e] = 0.0f;
          }
        }
        const float* nk = sN + s * 128 + j0;  // the column norms rk_j
        if (q4 < 2) {  // K row i: A_ij = beta_i rk_i rk_j e^{G_i - G_j} k_i.k_j
          const float bi = sbeta[s * CH + i] * sN[s * 128 + i];
#pragma unroll
          for (int j4 = 0; j4 < 8; j4++) {
            const float4 f = *reinterpret_cast<const float4*>(nk + 4 * j4);
            const float r4[4] = {f.x, f.y, f.z, f.w};
            float av[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const int jj = 4 * j4 + e;
              av[e] = j0 + jj < i ? bi * r4[e] * dec[jj] * __uint_as_float(v[jj]) : 0.0f;
            }
            *reinterpret_cast<float4*>(sa + i * LA + j0 + 4 * j4) = make_float4(av[0], av[1], av[2], av[3]);
          }
        } else {  // Q row i: its P columns (f16, P_ij = rq_i rk_j e^{G_i - G_j} q_i.k_j), then Gamma_i rq_i q_i
                  // over one half of the row
          uint8_t* pt_ = base + (s ? kOffP1 : kOffP0);
          const float rq = sN[s * 128 + 64 + i];
#pragma unroll
          for (int j8 = 0; j8 < 4; j8++) {
            const float4 f0 = *reinterpret_cast<const float4*>(nk + 8 * j8), f1 = *reinterpret_cast<const float4*>(nk + 8 * j8 + 4);
            const float r8[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
            float p[8];
#pragma unroll
            for (int e = 0; e < 8; e++) p[e] = rq * r8[e] * dec[j8 * 8 + e] * __uint_as_float(v[j8 * 8 + e]);
            *reinterpret_cast<uint4*>(pt_ + swz(i, 4 * colh + j8)) =
                make_uint4(pack_h2(p[0], p[1]), pack_h2(p[2], p[3]), pack_h2(p[4], p[5]), pack_h2(p[6], p[7]));
          }
          const __half2 ga = __float2half2_rn(sGam[i] * rq);  // (below f16's range: zero, as its terms)
          uint8_t* qb = t + colh * kBox;
          uint4 u[8];
#pragma unroll
          for (int j8 = 0; j8 < 8; j8++) u[j8] = *reinterpret_cast<const uint4*>(qb + swz(64 + i, j8));
#pragma unroll
          for (int j8 = 0; j8 < 8; j8++) {
            __half2* w = reinterpret_cast<__half2*>(&u[j8]);
#pragma unroll
            for (int e = 0; e < 4; e++) w[e] = __hmul2(w[e], ga);
            *reinterpret_cast<uint4*>(qb + swz(64 + i, j8)) = u[j8];
          }
        }
      }
      tc_fence_before();
      prep_sync();
      // (4) T = (I + A)^-1
      tri_inverse(sa, sy, pw, pt, lane);
      // (5) T1 = T diag(beta Gamma rk), T2 = T diag(beta) (f16), once U of chunk c - 1 has read T2 (and W
      // of chunk c - 1, issued before it, T1); thread pt: row pt >> 2, columns 16 (pt & 3) ..
      if (ok && c >= 1) ok = mbar_wait_warp<false>(&bar[B_U_DONE + (s ^ 1)], ((c - 1) >> 1) & 1, abort, err, kErrTimeoutEmpty);
      if (ok) {
        const int i = pt >> 2, j0 = (pt & 3) * 16;
        const float* be = sbeta + s * CH;
        float tv[16], bj[16], gj[16];  // loaded before any store (see the A and P loops)
#pragma unroll
        for (int j4 = 0; j4 < 4; j4++) {  // T is lower triangular: its entries above the diagonal are zeros
          const float4 f = *reinterpret_cast<const float4*>(sa + i * LA + j0 + 4 * j4);
          tv[4 * j4] = f.x, tv[4 * j4 + 1] = f.y, tv[4 * j4 + 2] = f.z, tv[4 * j4 + 3] = f.w;
        }
#pragma unroll
        for (int j4 = 0; j4 < 4; j4++) {
          const float4 f = *reinterpret_cast<const float4*>(be + j0 + 4 * j4);
          const float4 h = *reinterpret_cast<const float4*>(sGam + j0 + 4 * j4);
          const float4 nk = *reinterpret_cast<const float4*>(sN + s * 128 + j0 + 4 * j4);
          bj[4 * j4] = f.x, bj[4 * j4 + 1] = f.y, bj[4 * j4 + 2] = f.z, bj[4 * j4 + 3] = f.w;
          gj[4 * j4] = h.x * nk.x, gj[4 * j4 + 1] = h.y * nk.y, gj[4 * j4 + 2] = h.z * nk.z, gj[4 * j4 + 3] = h.w * nk.w;
        }
#pragma unroll
        for (int j8 = 0; j8 < 2; j8++) {
          float t1[8], t2[8];
#pragma unroll
          for (int e = 0; e < 8; e++) {
            const int k = j8 * 8 + e;
            t2[e] = tv[k] * bj[k];
            t1[e] = t2[e] * gj[k];  // Gamma_j rk_j (W = T diag(beta Gamma) K^ = T1 K)
          }
          const int pc = (j0 >> 3) + j8;
          *reinterpret_cast<uint4*>(base + kOffT1 + swz(i, pc)) =
              make_uint4(pack_h2(t1[0], t1[1]), pack_h2(t1[2], t1[3]), pack_h2(t1[4], t1[5]), pack_h2(t1[6], t1[7]));
          *reinterpret_cast<uint4*>(base + kOffT2 + swz(i, pc)) =
              make_uint4(pack_h2(t2[0], t2[1]), pack_h2(t2[2], t2[3]), pack_h2(t2[4], t2[5]), pack_h2(t2[6], t2[7]));
        }
      }
      fence_proxy_async_smem();
      prep_sync();
      if (pt == 0 && ok) {  // W = [T1; *] K^ into D_X[s], once the chain has read chunk c - 2's O out of it
        if (c >= 2) ok = mbar_wait<false>(&bar[B_O_READ + s], ((c >> 1) - 1) & 1, abort, err, kErrTimeoutEmpty);
        if (ok) {
          tc_fence_after();
          const uint64_t ad = sw128_desc(base + kOffT1), bd = sw128_mn_desc(t, kBox);
#pragma unroll
          for (int ks = 0; ks < 4; ks++) tc_mma_f16(dx, ad + (uint64_t)(2 * ks), bd + (uint64_t)(128 * ks), kIdB, ks > 0);
          tc_commit(&bar[B_W_FULL + s]);
          // the chain takes the chunk from here: -W out of W, then U and the state products
          mbar_arrive(&bar[B_WQ_READY + s]);
        }
      }
      tc_fence_before();
      // every preparation warp takes the same path through the barriers; a warp that gave up tells the others
      if (!__all_sync(0xffffffffu, ok)) *abort = 1;
      prep_sync();
      if (*abort) ok = false;
    }
    if (pt == 0) {
      tc_commit(&bar[B_END_PREP]);
      mbar_drain(&bar[B_END_PREP], 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // the walk of an empty sequence: the final state is the initial one
  if (nch == 0 && sout && warp < 4) {
    const int r = (warp & 3) * 32 + lane;
    for (int cv = 0; cv < DK; cv++) sout[(size_t)r * DK + cv] = sin ? sin[(size_t)r * DK + cv] : 0.0f;
  }
}

cudaError_t take_gdn_tc_err(int* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_gdn_tc_err, sizeof(int));
  const int zero = 0;
  if (e == cudaSuccess && *code != 0) e = cudaMemcpyToSymbol(g_gdn_tc_err, &zero, sizeof(int));
  return e;
}

cudaError_t preload_gdn_tc() {
  return cudaFuncSetAttribute(gdn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
}

cudaError_t launch_gdn_tc(const __half* q, const __half* k, int qk_stride, const __half* v, int v_stride, long long seq_qk,
                          long long seq_v, int rows, const GdnTcArgs& a, int walks, cudaStream_t st) {
  if (walks <= 0 || a.h <= 0 || rows <= 0 || qk_stride % 8 || v_stride % 8 || seq_qk % 8 || seq_v % 8 ||
      ((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)a.o) % 16 || (!a.seq_off && (a.l <= 0 || walks % a.h)))
    return cudaErrorInvalidValue;
  static bool attr[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> g(mu);
    if (!attr[dev]) {
      if ((e = preload_gdn_tc()) != cudaSuccess) return e;
      attr[dev] = true;
    }
  }
  const int zdim = a.seq_off ? 1 : walks / a.h;
  CUtensorMap qm, km, vm, om;
  // the outputs: rows of h * DK floats, one per token (packed: `rows` tokens; else walks / h sequences of l)
  const long long orows = a.seq_off ? (long long)rows : (long long)(walks / a.h) * a.l;
  if (make_map_3d(&qm, q, a.h * DK, rows, zdim, qk_stride, a.seq_off ? (long long)rows * qk_stride : seq_qk, CH) != 0 ||
      make_map_3d(&km, k, a.h * DK, rows, zdim, qk_stride, a.seq_off ? (long long)rows * qk_stride : seq_qk, CH) != 0 ||
      make_map_3d(&vm, v, a.h * DK, rows, zdim, v_stride, a.seq_off ? (long long)rows * v_stride : seq_v, CH) != 0 ||
      make_map_f32(&om, a.o, orows, a.h * DK, (long long)a.h * DK, 32) != 0)
    return cudaErrorInvalidValue;
  return launch_dependent(gdn_tc_kernel, dim3(walks), dim3(kThreads), kSmem, st, qm, km, vm, om, a);
}

}  // namespace sd
