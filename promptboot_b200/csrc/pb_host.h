// Host-side shared state of the library: CUDA error capture, the RoPE table,
// SHA-256 and the model handle.  Not part of the public C ABI.
#pragma once

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/promptboot_b200.h"

namespace pb {

// Records the failing CUDA call's text for pb_last_error_string() and returns
// PB_DEVICE.  Every CUDA runtime call on an ABI path goes through PB_CUDA.
uint32_t record_cuda_error(cudaError_t e, const char* what);
#define PB_CUDA(call)                                                    \
  do {                                                                   \
    cudaError_t pb_e_ = (call);                                          \
    if (pb_e_ != cudaSuccess) return ::pb::record_cuda_error(pb_e_, #call); \
  } while (0)

// Sets the text returned by pb_last_error_string() for a non-CUDA failure.
void set_last_error(const char* text);

void sha256(const uint8_t* data, size_t len, uint8_t out[32]);

// The 8 MiB inference RoPE table (tests/fixtures/inference/
// generate_inference_rope_fixture.py in the reference): glibc powf/cosf/sinf
// over a binary32 angle recurrence.  Returns false if its SHA-256 is not the
// reference's pinned cd75fcc6...c01c5 (a different libm on this host).
bool build_rope_table(std::vector<float>& table);

constexpr uint64_t kModelBytes = 426762944ull;
constexpr uint64_t kTensorSection = 3980480ull;   // section 7 offset
constexpr uint64_t kTensorDirectory = 3952512ull; // section 6 offset
constexpr uint64_t kTensorDataBytes = 422782464ull;

}  // namespace pb

struct pb_model {
  int device = 0;
  uint8_t* data = nullptr;           // device copy of section 7
  uint64_t offset[291] = {};         // file offsets of each tensor
  uint64_t length[291] = {};
  float* rope = nullptr;             // device RoPE table
  // Tensor-core tile image of every matvec weight (pb_gemm_tc.cu layout), per
  // layer [q|k|v] [o] [gate|up] [down] stacked by row tiles, then the output head.
  uint8_t* tc = nullptr;
  size_t tc_bytes = 0;
  size_t tc_qkv[24] = {}, tc_o[24] = {}, tc_gateup[24] = {}, tc_down[24] = {}, tc_head = 0;
  // Tile image of the Q4_0 token embedding used as a tied 896 -> 151936 output
  // head (pb_model_matvec_device on tensor 0), built on its first use.
  uint8_t* tc_embed = nullptr;
  // Scratch of pb_model_matvec_device (grown on demand) and its pipeline status word.
  uint8_t* op_scratch = nullptr;
  size_t op_scratch_bytes = 0;
  unsigned int* op_status = nullptr;
  const uint8_t* tensor(uint32_t id) const {
    return data + (offset[id] - pb::kTensorSection);
  }
};
