// Rotary position embedding of q and k in one launch (sm_100a), forward and backward.
//
// Reference: rope_pair_forward_kernel / rope_pair_backward_kernel
// (solution/kernels/rope.py:24-105, patch solution/rope.py:55-80).  For each
// (batch b, head h, token t) and column d < D/2, with x1 = x[d], x2 = x[d + D/2],
// c1 = cos[d], c2 = cos[d + D/2], s1 = sin[d], s2 = sin[d + D/2]:
//
//   forward   y[d]       = R(x1 * c1) + R(-x2 * s1)        R: round to the output dtype
//   (y dtype  y[d + D/2] = R(x2 * c2) + R(x1 * s2)            promote(x, cos))
//   backward  dx[d]       = R(g1 * c1) + R(g2 * s2)       R: round to x's dtype
//             dx[d + D/2] = R(g2 * c2) - R(g1 * s1)
//
// Every product is rounded to the destination dtype before the addition and the
// sum is rounded again on store -- eager PyTorch's `q * cos + rotate_half(q) * sin`
// and its autograd -- so the results are bit-identical to the reference for fp16
// and fp32 inputs.  Products and sums use explicit round-to-nearest intrinsics
// (no contraction into FMA).
//
// Layout: q [B, Hq, S, D] and k [B, Hk, S, D] with any strides (Qwen2 passes the
// transposed [B, S, H, D] projection view), cos/sin [1 or B, S, D]; outputs are
// contiguous [B, H, S, D].  The work is ordered (b, t, head, column chunk) so that
// the heads of one token -- adjacent in the projection's memory -- are read
// together and share the token's cos/sin row from L1.  HBM-bound: per token
// 2 x (Hq + Hk) x D elements read and written plus the cos/sin row.
#pragma once

#include "common.cuh"

namespace sb {
namespace rope {

struct Side {
  const void* src;   // forward: q or k; backward: the gradient of the output
  int src_dt;
  int64_t sb, sh, st, sd;  // element strides of src (batch, head, token, column)
  void* dst;         // contiguous [B, heads, S, D]
  int dst_dt;
  int64_t heads;
};

struct Args {
  Side side[2];            // 0: q, 1: k
  const void* cos;
  const void* sin;
  int cs_dt;
  int64_t cb, ct, sb_, st_;  // cos / sin strides (batch, token); unit column stride
  int64_t cs_batches;        // 1 (broadcast) or B
  int64_t batches, tokens, half;
  int backward;
};

template <int VEC>
__device__ __forceinline__ void load(const void* p, int dt, int64_t off, int64_t stride, float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    if (dt == SB_F32) {
      const float4 x = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + off);
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else {
      const uint2 x = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p) + off);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&x.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&x.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = ld_as_f32(p, dt, off + i * stride);
  }
}

template <int VEC>
__device__ __forceinline__ void store(void* p, int dt, int64_t off, const float (&v)[VEC]) {
  if constexpr (VEC == 4) {
    if (dt == SB_F32) {
      *reinterpret_cast<float4*>(static_cast<float*>(p) + off) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      __half2 a = __floats2half2_rn(v[0], v[1]);
      __half2 b = __floats2half2_rn(v[2], v[3]);
      uint2 x;
      x.x = *reinterpret_cast<uint32_t*>(&a);
      x.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(static_cast<__half*>(p) + off) = x;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) st_from_f32(p, dt, off + i, v[i]);
  }
}

// VEC columns per thread (4: every row, cos/sin and output offset is a multiple
// of 4 elements and the column stride is 1; 1 otherwise).
template <int VEC>
__global__ void __launch_bounds__(256) rope_kernel(const Args a) {
  const int64_t heads = a.side[0].heads + a.side[1].heads;
  const int64_t chunks = (a.half + VEC - 1) / VEC;
  const int64_t total = a.batches * a.tokens * heads * chunks;
  const int64_t width = 2 * a.half;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t chunk = w % chunks;
    int64_t rest = w / chunks;
    const int64_t head = rest % heads;
    rest /= heads;
    const int64_t t = rest % a.tokens;
    const int64_t b = rest / a.tokens;
    const int which = head < a.side[0].heads ? 0 : 1;
    const Side& sd = a.side[which];
    const int64_t h = which == 0 ? head : head - a.side[0].heads;
    const int64_t d0 = chunk * VEC;
    const int64_t cbatch = a.cs_batches == 1 ? 0 : b;
    const int64_t coff = cbatch * a.cb + t * a.ct + d0;
    const int64_t soff = cbatch * a.sb_ + t * a.st_ + d0;
    const int64_t xoff = b * sd.sb + h * sd.sh + t * sd.st + d0 * sd.sd;
    const int64_t yoff = ((b * sd.heads + h) * a.tokens + t) * width + d0;
    if (VEC == 1 && d0 >= a.half) continue;
    float c1[VEC], c2[VEC], s1[VEC], s2[VEC], x1[VEC], x2[VEC], lo[VEC], hi[VEC];
    load<VEC>(a.cos, a.cs_dt, coff, 1, c1);
    load<VEC>(a.cos, a.cs_dt, coff + a.half, 1, c2);
    load<VEC>(a.sin, a.cs_dt, soff, 1, s1);
    load<VEC>(a.sin, a.cs_dt, soff + a.half, 1, s2);
    load<VEC>(sd.src, sd.src_dt, xoff, sd.sd, x1);
    load<VEC>(sd.src, sd.src_dt, xoff + a.half * sd.sd, sd.sd, x2);
    const int dt = sd.dst_dt;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      if (!a.backward) {
        lo[i] = __fadd_rn(round_to(__fmul_rn(x1[i], c1[i]), dt), round_to(__fmul_rn(-x2[i], s1[i]), dt));
        hi[i] = __fadd_rn(round_to(__fmul_rn(x2[i], c2[i]), dt), round_to(__fmul_rn(x1[i], s2[i]), dt));
      } else {
        lo[i] = __fadd_rn(round_to(__fmul_rn(x1[i], c1[i]), dt), round_to(__fmul_rn(x2[i], s2[i]), dt));
        hi[i] = __fsub_rn(round_to(__fmul_rn(x2[i], c2[i]), dt), round_to(__fmul_rn(x1[i], s1[i]), dt));
      }
    }
    store<VEC>(sd.dst, dt, yoff, lo);
    store<VEC>(sd.dst, dt, yoff + a.half, hi);
  }
}

inline bool side_vec4(const Side& s, int64_t half) {
  if (s.heads == 0) return true;
  const size_t src_bytes = s.src_dt == SB_F32 ? 16 : 8;
  const size_t dst_bytes = s.dst_dt == SB_F32 ? 16 : 8;
  return s.sd == 1 && s.sb % 4 == 0 && s.sh % 4 == 0 && s.st % 4 == 0 && half % 4 == 0 &&
         aligned(s.src, src_bytes) && aligned(s.dst, dst_bytes);
}

inline int launch(const Args& a, void* stream) {
  const int64_t heads = a.side[0].heads + a.side[1].heads;
  if (a.batches == 0 || a.tokens == 0 || heads == 0 || a.half == 0) return SB_OK;
  const size_t cs_bytes = a.cs_dt == SB_F32 ? 16 : 8;
  const bool vec4 = side_vec4(a.side[0], a.half) && side_vec4(a.side[1], a.half) && a.cb % 4 == 0 &&
                    a.ct % 4 == 0 && a.sb_ % 4 == 0 && a.st_ % 4 == 0 && aligned(a.cos, cs_bytes) &&
                    aligned(a.sin, cs_bytes);
  const int vec = vec4 ? 4 : 1;
  const int64_t work = a.batches * a.tokens * heads * ((a.half + vec - 1) / vec);
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, cap));
  if (vec4) {
    rope_kernel<4><<<grid, 256, 0, as_stream(stream)>>>(a);
  } else {
    rope_kernel<1><<<grid, 256, 0, as_stream(stream)>>>(a);
  }
  count_launch();
  return check_launch("rope_kernel");
}

}  // namespace rope
}  // namespace sb

extern "C" {

int sb_rope(const void* q, int q_dtype, const int64_t* q_strides, int64_t q_heads, void* q_out,
            int q_out_dtype, const void* k, int k_dtype, const int64_t* k_strides, int64_t k_heads,
            void* k_out, int k_out_dtype, const void* cos, const void* sin, int cs_dtype,
            const int64_t* cos_strides, const int64_t* sin_strides, int64_t cs_batches,
            int64_t batches, int64_t tokens, int64_t dim, int backward, void* stream) {
  SB_REQUIRE(batches >= 0 && tokens >= 0 && q_heads >= 0 && k_heads >= 0, "negative size");
  SB_REQUIRE(dim > 0 && dim % 2 == 0, "the head dimension must be positive and even");
  SB_REQUIRE(cs_batches == 1 || cs_batches == batches, "cos/sin batch must be 1 or the batch");
  SB_REQUIRE(sb::dtype_ok(cs_dtype), "cos/sin dtype must be SB_F16 or SB_F32");
  SB_REQUIRE(cos && sin && cos_strides && sin_strides, "NULL cos/sin argument");
  sb::rope::Args a{};
  const void* srcs[2] = {q, k};
  void* dsts[2] = {q_out, k_out};
  const int64_t* strides[2] = {q_strides, k_strides};
  const int src_dt[2] = {q_dtype, k_dtype};
  const int dst_dt[2] = {q_out_dtype, k_out_dtype};
  const int64_t heads[2] = {q_heads, k_heads};
  for (int i = 0; i < 2; ++i) {
    sb::rope::Side& s = a.side[i];
    s.heads = heads[i];
    if (heads[i] == 0) continue;
    SB_REQUIRE(srcs[i] && dsts[i] && strides[i], "NULL q/k argument with heads > 0");
    SB_REQUIRE(sb::dtype_ok(src_dt[i]) && sb::dtype_ok(dst_dt[i]), "q/k dtype must be SB_F16 or SB_F32");
    s.src = srcs[i];
    s.dst = dsts[i];
    s.src_dt = src_dt[i];
    s.dst_dt = dst_dt[i];
    s.sb = strides[i][0];
    s.sh = strides[i][1];
    s.st = strides[i][2];
    s.sd = strides[i][3];
  }
  a.cos = cos;
  a.sin = sin;
  a.cs_dt = cs_dtype;
  a.cb = cos_strides[0];
  a.ct = cos_strides[1];
  SB_REQUIRE(cos_strides[2] == 1 && sin_strides[2] == 1, "cos/sin need a unit column stride");
  a.sb_ = sin_strides[0];
  a.st_ = sin_strides[1];
  a.cs_batches = cs_batches;
  a.batches = batches;
  a.tokens = tokens;
  a.half = dim / 2;
  a.backward = backward ? 1 : 0;
  return sb::rope::launch(a, stream);
}

}  // extern "C"
