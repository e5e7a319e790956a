// SwiGLU arithmetic of the Qwen2 MLP (sm_100a), shared by the element-wise kernels
// below and the epilogues of the fused gate/up and down GEMMs (gemm_pair.cuh).
//
// Reference: swiglu_tile_engine (solution/kernels/swiglu_fused.py:21-46), on the
// fp16 outputs of the gate / up projections, in fp32:
//
//   p  = 1 / (1 + exp(-g))        a  = (g * p) * u
//   dg = (da * u) * (p + (g p) (1 - p))        du = da * (g p)
//
// Each multiply and add is rounded separately (explicit _rn intrinsics, no
// contraction).  The exponential and the reciprocal are the fast hardware forms
// (__expf, __fdividef), the same approximation class as the reference's
// tl.exp and fp32 division on the GPU; their few-ulp fp32 error is far below the
// fp16 rounding of the results.
#pragma once

#include "common.cuh"

namespace sb {
namespace swiglu {

__device__ __forceinline__ float sigmoid(float g) { return __fdividef(1.0f, __fadd_rn(1.0f, __expf(-g))); }

__device__ __forceinline__ float forward(float g, float u) {
  return __fmul_rn(__fmul_rn(g, sigmoid(g)), u);
}

__device__ __forceinline__ void backward(float g, float u, float da, float& dg, float& du) {
  const float p = sigmoid(g);
  const float act = __fmul_rn(g, p);
  const float slope = __fadd_rn(p, __fmul_rn(act, __fsub_rn(1.0f, p)));
  dg = __fmul_rn(__fmul_rn(da, u), slope);
  du = __fmul_rn(da, act);
}

// Element-wise forms over fp16 [rows, width] matrices with row pitches (elements);
// eight columns per thread with 16-byte accesses when every pitch and pointer allows.
struct Mat {
  const __half* p;
  int64_t ld;
};

template <bool VEC8, bool BWD>
__global__ void __launch_bounds__(256) swiglu_kernel(Mat g, Mat u, Mat da, __half* out0, int64_t ld0,
                                                     __half* out1, int64_t ld1, int64_t rows, int64_t width) {
  constexpr int kV = VEC8 ? 8 : 1;
  const int64_t per_row = (width + kV - 1) / kV;
  const int64_t total = rows * per_row;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = w / per_row;
    const int64_t c = (w % per_row) * kV;
    alignas(16) __half gv[kV], uv[kV], dv[kV], o0[kV], o1[kV];
    if constexpr (VEC8) {
      *reinterpret_cast<uint4*>(gv) = *reinterpret_cast<const uint4*>(g.p + r * g.ld + c);
      *reinterpret_cast<uint4*>(uv) = *reinterpret_cast<const uint4*>(u.p + r * u.ld + c);
      if constexpr (BWD) *reinterpret_cast<uint4*>(dv) = *reinterpret_cast<const uint4*>(da.p + r * da.ld + c);
    } else {
      gv[0] = g.p[r * g.ld + c];
      uv[0] = u.p[r * u.ld + c];
      if constexpr (BWD) dv[0] = da.p[r * da.ld + c];
    }
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const float gf = __half2float(gv[i]), uf = __half2float(uv[i]);
      if constexpr (BWD) {
        float dg, du;
        backward(gf, uf, __half2float(dv[i]), dg, du);
        o0[i] = __float2half_rn(dg);
        o1[i] = __float2half_rn(du);
      } else {
        o0[i] = __float2half_rn(forward(gf, uf));
      }
    }
    if constexpr (VEC8) {
      *reinterpret_cast<uint4*>(out0 + r * ld0 + c) = *reinterpret_cast<const uint4*>(o0);
      if constexpr (BWD) *reinterpret_cast<uint4*>(out1 + r * ld1 + c) = *reinterpret_cast<const uint4*>(o1);
    } else {
      out0[r * ld0 + c] = o0[0];
      if constexpr (BWD) out1[r * ld1 + c] = o1[0];
    }
  }
}

inline bool vec8_ok(const void* p, int64_t ld) { return aligned(p, 16) && ld % 8 == 0; }

template <bool BWD>
inline int launch(Mat g, Mat u, Mat da, __half* out0, int64_t ld0, __half* out1, int64_t ld1, int64_t rows,
                  int64_t width, void* stream) {
  if (rows == 0 || width == 0) return SB_OK;
  bool v8 = width % 8 == 0 && vec8_ok(g.p, g.ld) && vec8_ok(u.p, u.ld) && vec8_ok(out0, ld0);
  if (BWD) v8 = v8 && vec8_ok(da.p, da.ld) && vec8_ok(out1, ld1);
  const int64_t work = rows * (v8 ? width / 8 : width);
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, cap));
  if (v8) {
    swiglu_kernel<true, BWD><<<grid, 256, 0, as_stream(stream)>>>(g, u, da, out0, ld0, out1, ld1, rows, width);
  } else {
    swiglu_kernel<false, BWD><<<grid, 256, 0, as_stream(stream)>>>(g, u, da, out0, ld0, out1, ld1, rows, width);
  }
  count_launch();
  return check_launch("swiglu_kernel");
}

}  // namespace swiglu
}  // namespace sb

extern "C" {

int sb_swiglu_fwd(const uint16_t* gate, int64_t ld_gate, const uint16_t* up, int64_t ld_up, uint16_t* act,
                  int64_t ld_act, int64_t rows, int64_t width, void* stream) {
  SB_REQUIRE(rows >= 0 && width >= 0, "negative size");
  if (rows == 0 || width == 0) return SB_OK;
  SB_REQUIRE(gate && up && act, "NULL pointer argument");
  SB_REQUIRE(ld_gate >= width && ld_up >= width && ld_act >= width, "row pitch below the width");
  using sb::swiglu::Mat;
  const __half* g = reinterpret_cast<const __half*>(gate);
  return sb::swiglu::launch<false>(Mat{g, ld_gate}, Mat{reinterpret_cast<const __half*>(up), ld_up}, Mat{g, 0},
                                   reinterpret_cast<__half*>(act), ld_act, nullptr, 0, rows, width, stream);
}

int sb_swiglu_bwd(const uint16_t* gate, int64_t ld_gate, const uint16_t* up, int64_t ld_up,
                  const uint16_t* grad, int64_t ld_grad, uint16_t* dgate, int64_t ld_dgate, uint16_t* dup,
                  int64_t ld_dup, int64_t rows, int64_t width, void* stream) {
  SB_REQUIRE(rows >= 0 && width >= 0, "negative size");
  if (rows == 0 || width == 0) return SB_OK;
  SB_REQUIRE(gate && up && grad && dgate && dup, "NULL pointer argument");
  SB_REQUIRE(ld_gate >= width && ld_up >= width && ld_grad >= width && ld_dgate >= width && ld_dup >= width,
             "row pitch below the width");
  using sb::swiglu::Mat;
  return sb::swiglu::launch<true>(Mat{reinterpret_cast<const __half*>(gate), ld_gate},
                                  Mat{reinterpret_cast<const __half*>(up), ld_up},
                                  Mat{reinterpret_cast<const __half*>(grad), ld_grad},
                                  reinterpret_cast<__half*>(dgate), ld_dgate, reinterpret_cast<__half*>(dup),
                                  ld_dup, rows, width, stream);
}

}  // extern "C"
