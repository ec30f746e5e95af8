// Test shim (C linkage) around the header-only packing of include/purin_cp_ffi.h,
// so the Python tests can drive it through ctypes without XLA or a GPU.
#include <cstring>
#include <string>

#include "purin_cp_ffi.h"

extern "C" {

int32_t shim_pack_forward(const PurinCpPlanInfo* info, const purin_ffi::ForwardBuffers* b,
                          int64_t sample_offset, int64_t total_batch, PurinCpForwardArgs* out,
                          char* message, int32_t message_size) {
  std::string m;
  const int32_t s = purin_ffi::pack_forward(*info, *b, sample_offset, total_batch, out, &m);
  std::strncpy(message, m.c_str(), (size_t)message_size - 1);
  message[message_size - 1] = 0;
  return s;
}

int32_t shim_pack_adjoint(const PurinCpPlanInfo* info, const purin_ffi::AdjointBuffers* b,
                          int64_t sample_offset, int64_t total_batch, PurinCpAdjointArgs* out,
                          char* message, int32_t message_size) {
  std::string m;
  const int32_t s = purin_ffi::pack_adjoint(*info, *b, sample_offset, total_batch, out, &m);
  std::strncpy(message, m.c_str(), (size_t)message_size - 1);
  message[message_size - 1] = 0;
  return s;
}

void shim_make_config(int64_t max_iterations, int32_t accelerated, double safety,
                      int64_t norm_iterations, int64_t norm_seed, int32_t norm_bound,
                      int32_t diagonal, int32_t partitionable, PurinCpConfig* out) {
  *out = purin_ffi::make_config(max_iterations, accelerated != 0, safety, norm_iterations,
                                norm_seed, norm_bound != 0, diagonal != 0, partitionable != 0);
}

}  // extern "C"
