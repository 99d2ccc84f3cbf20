// Single CUDA translation unit of libdsv4moe.so: the kernel files share one
// device-side error flag and the internal launchers, so they are compiled
// together.
#include "gate.cu"
#include "route.cu"
#include "expert_gemm.cu"
#include "expert_gemm_pair.cu"
#include "gate_gemm.cu"
#include "materialize.cu"
#include "ep.cu"
#include "sparse_attn.cu"
#include "capi.cu"
#include "no_alloc.cu"
