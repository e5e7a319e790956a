// Right-padding removal for one training batch (sm_100a): metadata, pack and scatter.
//
// Reference: solution/unpad.py -- _batch_metadata (:164-183: mask geometry and the
// padding-label check in one device-to-host transfer), _indices_from_lengths
// (:186-200: row-major positions of the real tokens), _pack (:149-150:
// index_select of the real rows into [1, T, ...]) and _scatter (:153-161: the
// packed rows written back into a zero [B, S, ...] buffer).
//
// Here:
//   unpad_rows_kernel   one CTA per batch row: counts the row's real tokens and
//                       checks that the mask is binary, right-padded and that every
//                       padded position's label is the ignore index;
//   unpad_offsets_kernel one CTA: exclusive prefix of the lengths -> cu_seqlens[B+1]
//                       (int32, the varlen-attention convention) and a validity word;
//   pack_rows_kernel    packed[i] = x[b, i - cu[b]] for the real rows (16-byte copies;
//                       the batch of packed row i is found by binary search in cu);
//   scatter_rows_kernel out[b, t] = packed[cu[b] + t] for t < len[b], zeros elsewhere
//                       (every output row written once: no separate zero fill).
// The host reads cu_seqlens and the validity word back in ONE copy (B + 2 int32).
// All memory-bound: pack reads and writes T rows, scatter writes B*S rows.
#pragma once

#include "common.cuh"

namespace sb {
namespace unpad {

enum : int { kBadValue = 1, kNotRightPadded = 2, kLabelOnPadding = 4, kEmptyRow = 8 };

// Mask element as 0 / 1 / other (-1), for int64, int32, uint8/bool, fp16 and fp32 masks.
__device__ __forceinline__ int mask_at(const void* mask, int mdt, int64_t i) {
  double v;
  switch (mdt) {
    case 0: v = static_cast<double>(static_cast<const int64_t*>(mask)[i]); break;
    case 1: v = static_cast<double>(static_cast<const int32_t*>(mask)[i]); break;
    case 2: v = static_cast<double>(static_cast<const uint8_t*>(mask)[i]); break;
    case 3: v = static_cast<double>(__half2float(static_cast<const __half*>(mask)[i])); break;
    default: v = static_cast<double>(static_cast<const float*>(mask)[i]); break;
  }
  return v == 0.0 ? 0 : (v == 1.0 ? 1 : -1);
}

__global__ void __launch_bounds__(256) unpad_rows_kernel(const void* mask, int mdt, const int64_t* labels,
                                                         int64_t ignore, int64_t seq, int32_t* lengths,
                                                         int32_t* flags) {
  const int64_t b = blockIdx.x;
  __shared__ int count_s, first_zero_s, last_one_s, bad_s;
  if (threadIdx.x == 0) {
    count_s = 0;
    first_zero_s = 0x7fffffff;
    last_one_s = -1;
    bad_s = 0;
  }
  __syncthreads();
  int count = 0, first_zero = 0x7fffffff, last_one = -1, bad = 0;
  for (int64_t t = threadIdx.x; t < seq; t += blockDim.x) {
    const int m = mask_at(mask, mdt, b * seq + t);
    if (m < 0) bad |= kBadValue;
    if (m == 1) {
      ++count;
      last_one = max(last_one, static_cast<int>(t));
    } else {
      first_zero = min(first_zero, static_cast<int>(t));
      if (labels && labels[b * seq + t] != ignore) bad |= kLabelOnPadding;
    }
  }
  atomicAdd(&count_s, count);
  atomicMin(&first_zero_s, first_zero);
  atomicMax(&last_one_s, last_one);
  atomicOr(&bad_s, bad);
  __syncthreads();
  if (threadIdx.x == 0) {
    int f = bad_s;
    if (last_one_s > first_zero_s) f |= kNotRightPadded;
    if (count_s == 0) f |= kEmptyRow;
    lengths[b] = count_s;
    if (f) atomicOr(flags, f);
  }
}

// cu[0..B] = exclusive prefix of lengths; cu[B + 1] = the validity flags.  One CTA.
__global__ void __launch_bounds__(1024) unpad_offsets_kernel(const int32_t* lengths, int64_t batch,
                                                             const int32_t* flags, int32_t* cu) {
  __shared__ int32_t carry;
  __shared__ int32_t warp_sums[32];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < batch; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    const int32_t v = i < batch ? lengths[i] : 0;
    // inclusive scan within the block
    int32_t x = v;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, d);
      if (lane >= d) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int32_t w = lane < static_cast<int>(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += y;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const int32_t before = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
    if (i < batch) cu[i] = before;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = before + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    cu[batch] = carry;
    cu[batch + 1] = *flags;
  }
}

__device__ __forceinline__ int64_t batch_of(const int32_t* cu, int64_t batch, int64_t row) {
  int64_t lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= row) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Rows of `width_bytes` bytes moved in 16-byte units (width_bytes % 16 == 0, aligned
// bases) or bytes otherwise.
template <bool VEC>
__global__ void __launch_bounds__(256) pack_rows_kernel(const uint8_t* x, int64_t seq, const int32_t* cu,
                                                        int64_t batch, int64_t rows, int64_t width_bytes,
                                                        uint8_t* packed) {
  const int64_t units = VEC ? width_bytes / 16 : width_bytes;
  const int64_t total = rows * units;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = w / units, u = w % units;
    const int64_t b = batch_of(cu, batch, row);
    const int64_t src_row = b * seq + (row - cu[b]);
    if constexpr (VEC) {
      reinterpret_cast<uint4*>(packed + row * width_bytes)[u] =
          reinterpret_cast<const uint4*>(x + src_row * width_bytes)[u];
    } else {
      packed[row * width_bytes + u] = x[src_row * width_bytes + u];
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(256) scatter_rows_kernel(const uint8_t* packed, int64_t seq, const int32_t* cu,
                                                           int64_t batch, int64_t width_bytes, uint8_t* out) {
  const int64_t units = VEC ? width_bytes / 16 : width_bytes;
  const int64_t total = batch * seq * units;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = w / units, u = w % units;
    const int64_t b = r / seq, t = r % seq;
    const bool real = t < static_cast<int64_t>(cu[b + 1] - cu[b]);
    const int64_t src = cu[b] + t;
    if constexpr (VEC) {
      reinterpret_cast<uint4*>(out + r * width_bytes)[u] =
          real ? reinterpret_cast<const uint4*>(packed + src * width_bytes)[u] : make_uint4(0, 0, 0, 0);
    } else {
      out[r * width_bytes + u] = real ? packed[src * width_bytes + u] : 0;
    }
  }
}

inline int grid_for(int64_t work) {
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  const int64_t g = (work + 255) / 256;
  return static_cast<int>(g < 1 ? 1 : (g < cap ? g : cap));
}

}  // namespace unpad
}  // namespace sb

extern "C" {

size_t sb_unpad_workspace_bytes(int64_t batch) {
  return static_cast<size_t>(batch + 1) * sizeof(int32_t);  // lengths + the flag word
}

int sb_unpad_metadata(const void* mask, int mask_dtype, const int64_t* labels, int64_t ignore_index, int64_t batch,
                      int64_t seq, int32_t* cu_seqlens, void* workspace, size_t workspace_bytes, void* stream) {
  SB_REQUIRE(batch >= 0 && seq >= 0 && seq < 0x7fffffffLL, "bad batch geometry");
  SB_REQUIRE(mask_dtype >= 0 && mask_dtype <= 4, "mask dtype code must be 0..4");
  SB_REQUIRE(cu_seqlens != nullptr, "NULL cu_seqlens");
  SB_REQUIRE(batch == 0 || mask != nullptr, "NULL mask");
  const size_t need = sb_unpad_workspace_bytes(batch);
  SB_REQUIRE(workspace && workspace_bytes >= need, "workspace smaller than sb_unpad_workspace_bytes");
  cudaStream_t st = sb::as_stream(stream);
  int32_t* lengths = static_cast<int32_t*>(workspace);
  int32_t* flags = lengths + batch;
  cudaError_t e = cudaMemsetAsync(flags, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return sb::fail(SB_ECUDA, std::string("flag reset: ") + cudaGetErrorString(e));
  if (batch > 0) {
    sb::unpad::unpad_rows_kernel<<<static_cast<unsigned>(batch), 256, 0, st>>>(mask, mask_dtype, labels,
                                                                              ignore_index, seq, lengths, flags);
    sb::count_launch();
    if (int rc = sb::check_launch("unpad_rows_kernel")) return rc;
  }
  sb::unpad::unpad_offsets_kernel<<<1, 1024, 0, st>>>(lengths, batch, flags, cu_seqlens);
  sb::count_launch();
  return sb::check_launch("unpad_offsets_kernel");
}

int sb_unpad_pack(const void* x, int64_t batch, int64_t seq, int64_t row_bytes, const int32_t* cu_seqlens,
                  int64_t rows, void* packed, void* stream) {
  SB_REQUIRE(batch >= 0 && seq >= 0 && row_bytes >= 0 && rows >= 0, "negative size");
  if (rows == 0 || row_bytes == 0) return SB_OK;
  SB_REQUIRE(x && cu_seqlens && packed && batch > 0, "NULL pointer argument");
  const bool vec = row_bytes % 16 == 0 && sb::aligned(x, 16) && sb::aligned(packed, 16);
  const int64_t work = rows * (vec ? row_bytes / 16 : row_bytes);
  cudaStream_t st = sb::as_stream(stream);
  if (vec) {
    sb::unpad::pack_rows_kernel<true><<<sb::unpad::grid_for(work), 256, 0, st>>>(
        static_cast<const uint8_t*>(x), seq, cu_seqlens, batch, rows, row_bytes, static_cast<uint8_t*>(packed));
  } else {
    sb::unpad::pack_rows_kernel<false><<<sb::unpad::grid_for(work), 256, 0, st>>>(
        static_cast<const uint8_t*>(x), seq, cu_seqlens, batch, rows, row_bytes, static_cast<uint8_t*>(packed));
  }
  sb::count_launch();
  return sb::check_launch("pack_rows_kernel");
}

int sb_unpad_scatter(const void* packed, int64_t batch, int64_t seq, int64_t row_bytes, const int32_t* cu_seqlens,
                     void* out, void* stream) {
  SB_REQUIRE(batch >= 0 && seq >= 0 && row_bytes >= 0, "negative size");
  if (batch == 0 || seq == 0 || row_bytes == 0) return SB_OK;
  SB_REQUIRE(packed && cu_seqlens && out, "NULL pointer argument");
  const bool vec = row_bytes % 16 == 0 && sb::aligned(packed, 16) && sb::aligned(out, 16);
  const int64_t work = batch * seq * (vec ? row_bytes / 16 : row_bytes);
  cudaStream_t st = sb::as_stream(stream);
  if (vec) {
    sb::unpad::scatter_rows_kernel<true><<<sb::unpad::grid_for(work), 256, 0, st>>>(
        static_cast<const uint8_t*>(packed), seq, cu_seqlens, batch, row_bytes, static_cast<uint8_t*>(out));
  } else {
    sb::unpad::scatter_rows_kernel<false><<<sb::unpad::grid_for(work), 256, 0, st>>>(
        static_cast<const uint8_t*>(packed), seq, cu_seqlens, batch, row_bytes, static_cast<uint8_t*>(out));
  }
  sb::count_launch();
  return sb::check_launch("scatter_rows_kernel");
}

}  // extern "C"
