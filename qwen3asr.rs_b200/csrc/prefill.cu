// prefill.cu — causal varlen (chunked) prefill attention over the pages.
#include "common.cuh"
#include "launch.h"

namespace vasr {

int launch_prefill(const PrefillArgs &a, cudaStream_t s) {
  (void)a;
  (void)s;
  return VASR_PA_ENOT_SUPPORTED;
}

int read_error_prefill(uint32_t *bits, bool clear, cudaStream_t s) {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_device_error, sizeof(v), 0, cudaMemcpyDeviceToHost, s) !=
      cudaSuccess)
    return VASR_PA_ELAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return VASR_PA_ELAUNCH;
  if (clear) {
    const uint32_t z = 0;
    if (cudaMemcpyToSymbolAsync(g_device_error, &z, sizeof(z), 0, cudaMemcpyHostToDevice, s) !=
        cudaSuccess)
      return VASR_PA_ELAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return VASR_PA_ELAUNCH;
  }
  *bits = v;
  return VASR_PA_OK;
}

}  // namespace vasr
