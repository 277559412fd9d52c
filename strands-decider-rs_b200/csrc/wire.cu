// The model's packed wire format, unpacked on the device at load (`src/model.rs:205-283`): 8-bit scale
// codes decoded to fp16 (`decode_scales`), packed shards laid out as the kernels read them
// (`unpack_shard`), embedding rows split into their parts (`embed_parts`). The power table
// 2^(-i / 4096) is built on the host with the same f64 `pow` as the reference's `Pow::upto`, so every
// decoded scale is bit-identical to the host decode.
#include <cmath>
#include <vector>

#include "common.cuh"
#include "sd_internal.h"

namespace sd {

namespace {

__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// Scale (r, i): header of row r at hdr + r hdr_stride (m as fp16 bits, then j as u16, little
// endian), code at codes + r code_stride + i; |scale| = fp16(f32(m pow[k j])), bit 7 of the code the
// sign.
__global__ void decode_scales_kernel(const uint8_t* __restrict__ hdr, size_t hdr_stride, const uint8_t* __restrict__ codes,
                                     size_t code_stride, long long n, int g, const double* __restrict__ pow,
                                     uint16_t* __restrict__ dst, size_t dst_stride) {
  const long long total = n * g;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (long long)gridDim.x * blockDim.x) {
    const long long r = t / g;
    const int i = (int)(t - r * g);
    const uint8_t* h = hdr + r * hdr_stride;
    const double m = (double)__half2float(__ushort_as_half(ld_u16(h)));
    const int j = ld_u16(h + 2);
    const uint8_t c = codes[r * code_stride + i];
    const uint16_t mag = __half_as_ushort(__float2half_rn((float)(m * pow[(c & 127) * j])));
    dst[r * dst_stride + i] = (uint16_t)(mag | ((uint16_t)(c & 128) << 8));
  }
}

// Bytes [off, off + len) of each of n rows of `stride` bytes to a dense [n][len] array.
__global__ void split_rows_kernel(const uint8_t* __restrict__ src, size_t stride, size_t off, size_t len, long long n,
                                  uint8_t* __restrict__ dst) {
  const long long total = n * (long long)len;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (long long)gridDim.x * blockDim.x) {
    const long long r = t / (long long)len;
    dst[t] = src[r * stride + off + (size_t)(t - r * (long long)len)];
  }
}

int grid_for(long long work) {
  const long long b = (work + 255) / 256;
  return (int)std::max<long long>(1, std::min<long long>(b, 148 * 16));
}

}  // namespace

cudaError_t decode_scales_dev(const uint8_t* hdr, size_t hdr_stride, const uint8_t* codes, size_t code_stride, long long n,
                              int g, int jmax, uint16_t* dst, size_t dst_stride, cudaStream_t st) {
  if (n <= 0 || g <= 0) return cudaSuccess;
  // 2^(-i / 4096) for every k j the codes can name (`Pow::upto`, src/model.rs:205-215)
  std::vector<double> table((size_t)127 * jmax + 1);
  for (size_t i = 0; i < table.size(); i++) table[i] = std::pow(2.0, -(double)i / 4096.0);
  double* dp = nullptr;
  cudaError_t e = cudaMallocAsync(&dp, table.size() * sizeof(double), st);
  if (e != cudaSuccess) return e;
  if ((e = cudaMemcpyAsync(dp, table.data(), table.size() * sizeof(double), cudaMemcpyHostToDevice, st)) == cudaSuccess) {
    decode_scales_kernel<<<grid_for(n * g), 256, 0, st>>>(hdr, hdr_stride, codes, code_stride, n, g, dp, dst, dst_stride);
    e = cudaGetLastError();
  }
  cudaFreeAsync(dp, st);
  // `table` is pageable: the copy out of it is staged before cudaMemcpyAsync returns
  return e;
}

cudaError_t split_rows_dev(const uint8_t* src, size_t stride, size_t off, size_t len, long long n, uint8_t* dst,
                           cudaStream_t st) {
  if (n <= 0 || len == 0) return cudaSuccess;
  split_rows_kernel<<<grid_for(n * (long long)len), 256, 0, st>>>(src, stride, off, len, n, dst);
  return cudaGetLastError();
}

}  // namespace sd
