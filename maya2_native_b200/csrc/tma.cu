// The driver's tensor-map encoder, resolved once per process (the runtime exposes driver entry points without
// linking libcuda directly).
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "tma.cuh"

namespace m3 {

namespace {
EncodeTiled g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int tensor_map_encoder(EncodeTiled* out) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiled>(fn);
  });
  M3_REQUIRE(g_encode, M3_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  *out = g_encode;
  return M3_OK;
}

}  // namespace m3
