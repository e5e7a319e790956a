// Standalone NF4 decode (bit-exact with the reference decoder).
//
// Reference: nf4_decode_kernel, solution/kernels/nf4.py:41-59; launched by
// dequantize_nf4 (:190-203, nested statistics) and _dequantize_flat_into
// (:181-187, fp32 absmax already rebuilt by bitsandbytes).
//
//   scale(b) = fp32(fp32(code2[qabs[b]] * absmax2[b >> 8]) + offset)   (nested)
//            = absmax[b]                                              (flat)
//   out[i]   = fp16_rn(NF4[nibble(i)] * scale(i >> 6))
//
// __fmul_rn / __fadd_rn keep the multiply and add separate (no FMA
// contraction), as the reference's enable_fp_fusion=False does.
//
// HBM-bound: 0.5 B read + 2 B written per element.  The vector path gives each
// thread one 32-bit word of packed nibbles (8 elements) and one 16-byte store,
// so a warp moves 128 B in and 512 B out per instruction, fully coalesced.
// The 16-entry NF4 table sits in shared memory: 16 words in 16 distinct banks,
// so any lookup pattern is conflict-free.  Unaligned views and tails take a
// one-element-per-thread path.
#pragma once

#include "common.cuh"

namespace sb {

__constant__ float c_nf4_values[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

struct ScaleSource {
  const uint8_t* qabs;
  const float* absmax2;
  const float* code2;
  const float* offset;
  const float* flat;  // non-null: flat fp32 absmax per block
};

__device__ __forceinline__ float block_scale(const ScaleSource& s, int64_t blk, float off) {
  if (s.flat) return __ldg(s.flat + blk);
  const float code = __ldg(s.code2 + __ldg(s.qabs + blk));
  const float second = __ldg(s.absmax2 + (blk >> 8));
  return __fadd_rn(__fmul_rn(code, second), off);
}

__global__ void __launch_bounds__(256) nf4_dequant_vec_kernel(const uint32_t* __restrict__ packed,
                                                              ScaleSource src,
                                                              uint4* __restrict__ out,
                                                              int64_t groups) {
  __shared__ float table[16];
  if (threadIdx.x < 16) table[threadIdx.x] = c_nf4_values[threadIdx.x];
  __syncthreads();
  const float off = src.flat ? 0.0f : __ldg(src.offset);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
       g += stride) {
    const uint32_t w = __ldg(packed + g);
    const float scale = block_scale(src, g >> 3, off);
    uint32_t res[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t byte = (w >> (8 * j)) & 0xFFu;
      const float hi = __fmul_rn(table[byte >> 4], scale);   // element 2j   (earlier)
      const float lo = __fmul_rn(table[byte & 15u], scale);  // element 2j+1
      __half2 h = __floats2half2_rn(hi, lo);
      res[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    out[g] = make_uint4(res[0], res[1], res[2], res[3]);
  }
}

__global__ void __launch_bounds__(256) nf4_dequant_scalar_kernel(const uint8_t* __restrict__ packed,
                                                                 ScaleSource src,
                                                                 __half* __restrict__ out,
                                                                 int64_t begin, int64_t n) {
  __shared__ float table[16];
  if (threadIdx.x < 16) table[threadIdx.x] = c_nf4_values[threadIdx.x];
  __syncthreads();
  const float off = src.flat ? 0.0f : __ldg(src.offset);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = begin + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    const uint32_t byte = __ldg(packed + (i >> 1));
    const uint32_t nib = (i & 1) ? (byte & 15u) : (byte >> 4);
    out[i] = __float2half_rn(__fmul_rn(table[nib], block_scale(src, i >> 6, off)));
  }
}

inline int launch_nf4_dequant(const uint8_t* packed, const ScaleSource& src, uint16_t* out,
                              int64_t n, cudaStream_t stream) {
  if (n == 0) return SB_OK;
  const int sms = device_sm_count();
  int64_t vec_groups = 0;
  if (aligned(packed, 4) && aligned(out, 16)) vec_groups = n / 8;
  if (vec_groups > 0) {
    const int64_t blocks = (vec_groups + 255) / 256;
    const int grid = static_cast<int>(blocks < sms * 16 ? blocks : sms * 16);
    nf4_dequant_vec_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const uint32_t*>(packed),
                                                     src, reinterpret_cast<uint4*>(out),
                                                     vec_groups);
    count_launch();
    if (int rc = check_launch("nf4_dequant_vec_kernel")) return rc;
  }
  const int64_t begin = vec_groups * 8;
  if (begin < n) {
    const int64_t rem = n - begin;
    const int64_t blocks = (rem + 255) / 256;
    const int grid = static_cast<int>(blocks < sms * 16 ? blocks : sms * 16);
    nf4_dequant_scalar_kernel<<<grid, 256, 0, stream>>>(packed, src,
                                                        reinterpret_cast<__half*>(out), begin, n);
    count_launch();
    if (int rc = check_launch("nf4_dequant_scalar_kernel")) return rc;
  }
  return SB_OK;
}

}  // namespace sb

extern "C" {

int sb_nf4_dequant_nested(const uint8_t* packed, const uint8_t* qabs, const float* absmax2,
                          const float* code2, const float* offset, uint16_t* out, int64_t n,
                          void* stream) {
  SB_REQUIRE(n >= 0, "n must be non-negative");
  if (n == 0) return SB_OK;
  SB_REQUIRE(packed && qabs && absmax2 && code2 && offset && out, "NULL pointer argument");
  sb::ScaleSource src{qabs, absmax2, code2, offset, nullptr};
  return sb::launch_nf4_dequant(packed, src, out, n, sb::as_stream(stream));
}

int sb_nf4_dequant_flat(const uint8_t* packed, const float* absmax, uint16_t* out, int64_t n,
                        void* stream) {
  SB_REQUIRE(n >= 0, "n must be non-negative");
  if (n == 0) return SB_OK;
  SB_REQUIRE(packed && absmax && out, "NULL pointer argument");
  sb::ScaleSource src{nullptr, nullptr, nullptr, nullptr, absmax};
  return sb::launch_nf4_dequant(packed, src, out, n, sb::as_stream(stream));
}

}  // extern "C"
