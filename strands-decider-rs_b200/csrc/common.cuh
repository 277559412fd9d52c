// Device-side helpers shared by the sm_100a kernels: bounded mbarrier waits, TMA and bulk copies,
// tcgen05 (TMEM allocation, MMA, commit, loads) and the int4 -> f16 dequantisation.
//
// Every wait on a barrier is bounded by wall time (globaltimer): a wait that runs out records an
// error code in the caller's error word and returns false, so a kernel with a bug ends instead of
// hanging the GPU. Host code reads the error word after the launch and fails the call.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sd_internal.h"

#define SD_DEV __device__ __forceinline__

namespace sd {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

SD_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

SD_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// The first 1024-byte aligned address at or after p, for p in shared memory. It is p plus an offset
// (not an integer round trip) so that the compiler still knows the result, and every pointer made
// from it, to be shared memory: it then emits shared loads and stores instead of generic ones, which
// take the longer path through the L1 and the long scoreboard.
SD_DEV uint8_t* smem_align1024(uint8_t* p) { return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u); }

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
SD_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
SD_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
SD_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
SD_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Tests the phase with parity `parity`; while it is not complete the thread is suspended in hardware
// (for at most kSuspendNs, woken when the phase completes), so waiting warps take no issue slots
// from the warps that share their scheduler (the MMA issuer above all). With `hint` false the
// suspension is the hardware's own short time limit: measured on B200, the GEMM is 3-9 % faster with
// the hint (its producers wait long and share schedulers with the dequantizing warps), attention 5 %
// and the gated-delta scan 1 % faster without (their waits are short and on their critical paths).
constexpr uint32_t kSuspendNs = 20000;
template <bool kHint = true>
SD_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if (kHint)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendNs)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  return ok != 0;
}

// Waits for the phase with parity `parity` to complete. Gives up after kWaitLimitNs, or soon after
// another thread of the CTA has given up (*abort set): records `code` in *err and returns false. Each
// poll sleeps in hardware until the phase completes (or kSuspendNs), then the clock and the abort flag
// are read.
template <bool kHint = true>
SD_DEV bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code, unsigned long long limit_ns) {
  if (mbar_try_wait<kHint>(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (true) {
    if (mbar_try_wait<kHint>(bar, parity)) return true;
    if (*abort) return false;
    if (global_ns() - t0 > limit_ns) {
      *abort = 1;
      atomicCAS(err, 0, code);
      return false;
    }
  }
}
template <bool kHint = true>
SD_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  return mbar_wait_for<kHint>(bar, parity, abort, err, code, kWaitLimitNs);
}

// mbar_wait for a whole warp: every lane polls (one try_wait instruction for the warp), so each
// lane has the barrier's acquire ordering. The lanes leave together: a lane that gave up (timeout or
// abort) makes the whole warp give up.
template <bool kHint = true>
SD_DEV bool mbar_wait_warp_for(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code,
                               unsigned long long limit_ns) {
  const bool ok = mbar_wait_for<kHint>(bar, parity, abort, err, code, limit_ns);
  return __all_sync(0xffffffffu, ok);
}
template <bool kHint = true>
SD_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  return mbar_wait_warp_for<kHint>(bar, parity, abort, err, code, kWaitLimitNs);
}

// Waits (bounded, ignoring the abort flag) for a phase that asynchronous copies or MMAs this CTA
// issued will complete, before the CTA exits: used on the way out, after an abort too, so that no
// copy lands in shared memory and no MMA writes TMEM after the CTA has released them.
SD_DEV void mbar_drain(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) return;
  }
}

// ---------------------------------------------------------------------------------------------
// TMA (no multicast: every CTA fetches its own tiles) and bulk copies
// ---------------------------------------------------------------------------------------------
SD_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
SD_DEV void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
SD_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// A tiled store from shared memory (the box of the map at x, y) into global memory, in the issuing
// thread's bulk group; the coordinates must lie inside the tensor (x a multiple of 16 bytes).
SD_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
SD_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the thread's committed bulk groups have read their shared memory (it may be written again)
SD_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// the thread's committed bulk groups have completed (their global writes are done)
SD_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
SD_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Programmatic dependent launch: a kernel launched with programmatic stream serialization may start
// while the kernel before it in the stream is still running; this waits until that kernel has
// completed and its memory operations are visible (a no-op for a kernel launched without it).
SD_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Launches `kern` with programmatic stream serialization (it may be scheduled while the kernel before
// it in `st` finishes: its launch, and whatever it does before grid_dep_wait, overlap that kernel's
// tail). Every kernel launched this way calls grid_dep_wait before it touches memory that earlier work
// in the stream writes or reads.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}
SD_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------------------------
SD_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
}
SD_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
SD_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
SD_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SD_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (f16 operands, f32 accumulate).
SD_DEV void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on `bar` once every MMA this thread issued before has completed.
SD_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
SD_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
SD_DEV void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A (M rows = TMEM lanes, K packed two f16 per
// 32-bit column) read from tensor memory.
SD_DEV void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers: thread i of the warp writes lane
// (base lane + i). Asynchronous: tc_wait_st before the data is signalled to another thread.
SD_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
SD_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
SD_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte swizzle:
// rows of 128 bytes (64 f16), 8-row groups 1024 bytes apart.
SD_DEV uint64_t sw128_desc(const void* smem_tile) {
  uint64_t addr = smem_u32(smem_tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;          // start address
  d |= (uint64_t)1 << 16;                // leading byte offset (unused with swizzle)
  d |= (uint64_t)(1024 >> 4) << 32;      // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                // SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor for an MN-major operand tile stored with the 128-byte swizzle: each
// row (one k) holds 64 consecutive f16 of the M or N dimension, 8-row groups are 1024 bytes apart, and
// the next 64 of M or N start `lbo_bytes` further on.
SD_DEV uint64_t sw128_mn_desc(const void* smem_tile, uint32_t lbo_bytes) {
  uint64_t addr = smem_u32(smem_tile);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;                      // start address
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;  // leading byte offset: next 64 of M or N
  d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset: next 8 rows of K
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                            // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: f16 A and B (K-major), f32 accumulator, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// The same with B MN-major (B stored k rows of N values).
__host__ __device__ constexpr uint32_t idesc_f16_bmn(int m, int n) { return idesc_f16(m, n) | (1u << 16); }

// ---------------------------------------------------------------------------------------------
// int4 dequantisation. Weight words are stored with the even elements of an 8-element group in
// the low 16 bits and the odd ones in the high 16 bits (repacked at load), so
// ((w >> 4i) & 0x000f000f) is the code pair (2i, 2i+1). (q + 1024) is exact in f16, so
// (q + 1024) - 1032 = q - 8 exactly, and the product with the scale rounds once, as the
// reference's `(f16(q) - 8.0) * sc` does.
// ---------------------------------------------------------------------------------------------
SD_DEV __half2 dq_pair(uint32_t w, int i, __half2 scale2) {
  uint32_t t = ((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u;
  __half2 v = *reinterpret_cast<__half2*>(&t);
  v = __hsub2(v, __half2half2(__ushort_as_half((unsigned short)0x6408)));  // 1032.0
  return __hmul2(v, scale2);
}

// The asymmetric format's pair: fma(q, scale, bias) in f16, one rounding, as the reference's
// `fma(vec4<f16>(q), sc, bi)` (src/kernels.rs:572); (q + 1024) - 1024 = q exactly.
SD_DEV __half2 dq_pair_affine(uint32_t w, int i, __half2 scale2, __half2 bias2) {
  uint32_t t = ((w >> (4 * i)) & 0x000F000Fu) | 0x64006400u;
  __half2 v = *reinterpret_cast<__half2*>(&t);
  v = __hsub2(v, __half2half2(__ushort_as_half((unsigned short)0x6400)));  // 1024.0
  return __hfma2(v, scale2, bias2);
}

SD_DEV uint32_t h2_as_u32(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }

SD_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
SD_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace sd
