// Test harness: the GPU kernels' per-lane GGUF dequant (kaggle-llm-endpoint_b200/csrc/iqlane.cuh) compiled for the
// host, so tests/test_iqlane_host.py can check its index and rounding logic against the oracle without a GPU.
// Built by that test with nvcc (host code only, -ffp-contract=off so no product is fused on the host either).
#include <cstdint>

#include "iqlane.cuh"

template <int T>
static void run(const uint8_t* blocks, long n_blocks, const float* table, float* out) {
  for (long b = 0; b < n_blocks; ++b)
    for (int lane = 0; lane < 32; ++lane) {
      float v[8];
      cbmoe::iq_lane8<T>(blocks + b * cbmoe::IqFmt<T>::kBytes, lane, table, v);
      for (int j = 0; j < 8; ++j) out[b * 256 + 8 * lane + j] = v[j];
    }
}

extern "C" int iqlane_host_dequant(int type, const uint8_t* blocks, long n_blocks, const float* table, float* out) {
  switch (type) {
    case CBMOE_GGML_IQ2_S: run<CBMOE_GGML_IQ2_S>(blocks, n_blocks, table, out); return 0;
    case CBMOE_GGML_IQ3_S: run<CBMOE_GGML_IQ3_S>(blocks, n_blocks, table, out); return 0;
    case CBMOE_GGML_IQ4_XS: run<CBMOE_GGML_IQ4_XS>(blocks, n_blocks, table, out); return 0;
    case CBMOE_GGML_Q2_K: run<CBMOE_GGML_Q2_K>(blocks, n_blocks, table, out); return 0;
    case CBMOE_GGML_Q3_K: run<CBMOE_GGML_Q3_K>(blocks, n_blocks, table, out); return 0;
    default: return -1;
  }
}
