// Unity build of libsoupsuck_b200.so: every component is one translation unit,
// so the device error word and constant tables need no relocatable device code.
#include "runtime.cuh"
#include "nf4_dequant.cuh"
#include "rowwise.cuh"
#include "gemm_sm100.cuh"
#include "gemm_host.cuh"
#include "linear.cuh"
#include "lora_mma.cuh"
#include "lora_static.cuh"
#include "cross_entropy.cuh"
#include "rope.cuh"
#include "swiglu.cuh"
#include "mlp.cuh"
