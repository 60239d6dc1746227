// std_b200.cu -- the single translation unit of libstd_b200.so.
//
// All kernels are compiled together so that the library-wide device error
// word (g_std_error, common.cuh) has one definition without relocatable
// device code.  Build: std_b200/build.py (nvcc -gencode
// arch=compute_100a,code=sm_100a -shared).
#include "common.cuh"

#include "decode_ops.cu"
#include "draft_attn.cu"
#include "merge.cu"
#include "p2p.cu"
#include "select.cu"
#include "verify_attn.cu"
#include "gemm.cu"
#include "graph_loop.cu"
#include "collect.cu"

extern "C" int std_version(void) { return 100; }

extern "C" int std_get_device_error(int* code_out) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_std_error, sizeof(int)) != cudaSuccess) return 4;
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_std_error, &zero, sizeof(int)) != cudaSuccess) return 4;
  if (code_out != nullptr) *code_out = v;
  return 0;
}

extern "C" int std_device_supported(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return 0;
  return (major == 10 && minor == 0) ? 1 : 0;
}
