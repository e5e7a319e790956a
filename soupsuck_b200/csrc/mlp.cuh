// C ABI of the fused Qwen2 MLP path on the 2-SM NF4 GEMM (gemm_host.cuh drivers).
//
// Reference: the frozen MLP boundary solution/mlp.py:500-593 -- gate/up
// projections, swiglu_fused_forward, down projection; backward: down dX,
// swiglu_fused_backward, gate/up dX summed -- with the SwiGLU tile engine
// solution/kernels/swiglu_fused.py:21-78.  Here the element-wise SwiGLU passes
// live in GEMM epilogues and the two gate/up input gradients are one reduction.
#pragma once

#include "common.cuh"
#include "gemm_host.cuh"

namespace sb {

inline int check_weight(const sb_nf4_weight* w) {
  SB_REQUIRE(w != nullptr, "NULL weight descriptor");
  SB_REQUIRE(w->n_out > 0 && w->k_in > 0, "empty weight");
  SB_REQUIRE(w->packed && w->qabs && w->absmax2 && w->code2 && w->offset, "NULL weight buffer");
  SB_REQUIRE(aligned(w->packed, 16), "packed codes must be 16-byte aligned");
  SB_REQUIRE(w->k_in % 64 == 0, "weight rows must hold whole 64-element blocks");
  SB_REQUIRE(w->n_out <= 0x7fffffffLL && w->k_in <= 0x7fffffffLL, "weight too large");
  return SB_OK;
}

inline int check_lora(int r, const void* a, const void* b) {
  SB_REQUIRE(r == 0 || r == 16 || r == 32 || r == 64, "LoRA rank must be 0, 16, 32 or 64");
  SB_REQUIRE(r == 0 || (a && b && aligned(a, 16) && aligned(b, 16)), "LoRA factors missing or misaligned");
  return SB_OK;
}

}  // namespace sb

extern "C" {

int sb_nf4_mlp_gate_up_fwd(const uint16_t* x, int64_t m, const sb_nf4_weight* gate, const sb_nf4_weight* up,
                           const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* gate_up,
                           uint16_t* act, void* stream) {
  if (int rc = sb::check_weight(gate)) return rc;
  if (int rc = sb::check_weight(up)) return rc;
  if (int rc = sb::check_lora(r, lora_a, lora_b)) return rc;
  SB_REQUIRE(sb::gemm::same_shape(*gate, *up), "gate and up weights must have the same shape");
  SB_REQUIRE(gate->n_out % 128 == 0, "the intermediate size must be a multiple of 128");
  SB_REQUIRE(m >= 0 && m <= 0x7fffffffLL, "row count out of range");
  if (m == 0) return SB_OK;
  SB_REQUIRE(x && gate_up && act, "NULL pointer argument");
  SB_REQUIRE(sb::aligned(x, 16) && sb::aligned(gate_up, 16) && sb::aligned(act, 16), "operands must be 16-byte aligned");
  return sb::gemm::mlp_gate_up(x, m, *gate, *up, lora_a, lora_b, r, gate_up, act, sb::as_stream(stream));
}

int sb_nf4_mlp_down_dx(const uint16_t* dy, int64_t m, const sb_nf4_weight* down, const uint16_t* lora_a,
                       const uint16_t* lora_b, int r, const uint16_t* gate_up, uint16_t* dgate_up, void* stream) {
  if (int rc = sb::check_weight(down)) return rc;
  if (int rc = sb::check_lora(r, lora_a, lora_b)) return rc;
  SB_REQUIRE(down->k_in % 64 == 0 && down->n_out % 8 == 0, "down weight shape not supported");
  SB_REQUIRE(m >= 0 && m <= 0x7fffffffLL, "row count out of range");
  if (m == 0) return SB_OK;
  SB_REQUIRE(dy && gate_up && dgate_up, "NULL pointer argument");
  SB_REQUIRE(sb::aligned(dy, 16) && sb::aligned(gate_up, 16) && sb::aligned(dgate_up, 16),
             "operands must be 16-byte aligned");
  return sb::gemm::mlp_down_dx(dy, m, *down, lora_a, lora_b, r, gate_up, dgate_up, sb::as_stream(stream));
}

size_t sb_nf4_linear_dx2_workspace_bytes(int64_t m, int64_t n_out, int64_t k_in) {
  if (m <= 0 || n_out <= 0 || k_in <= 0) return 0;
  return sb::gemm::dx2_plan(m, n_out, k_in).workspace;
}

int sb_nf4_linear_dx2(const uint16_t* dy2, int64_t m, const sb_nf4_weight* w1, const sb_nf4_weight* w2,
                      const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* dx, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (int rc = sb::check_weight(w1)) return rc;
  if (int rc = sb::check_weight(w2)) return rc;
  if (int rc = sb::check_lora(r, lora_a, lora_b)) return rc;
  SB_REQUIRE(sb::gemm::same_shape(*w1, *w2), "the two weights must have the same shape");
  SB_REQUIRE(w1->n_out % 64 == 0, "each weight's output size must be a multiple of 64");
  SB_REQUIRE(m >= 0 && m <= 0x7fffffffLL, "row count out of range");
  if (m == 0) return SB_OK;
  SB_REQUIRE(dy2 && dx, "NULL pointer argument");
  SB_REQUIRE(sb::aligned(dy2, 16) && sb::aligned(dx, 16), "operands must be 16-byte aligned");
  return sb::gemm::linear_dx2(dy2, m, *w1, *w2, lora_a, lora_b, r, dx, workspace, workspace_bytes,
                              sb::as_stream(stream));
}

}  // extern "C"
