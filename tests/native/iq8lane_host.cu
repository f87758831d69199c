// Test harness: the transcode and A-fragment arithmetic of the int8 GGUF kernels (csrc/iq8lane.cuh) compiled for
// the host. For 16 rows of one raw block each it builds every lane's words, turns them into the MMA A fragments the
// kernel builds, places each fragment byte at the (row, input) the MMA gives it, and returns value x group factor x
// block scale per weight, which tests/test_iq8lane_host.py compares bit for bit with the oracle's dequant. It also
// checks that the activations' storage order puts each B byte at the input its A byte multiplies.
#include <cstdint>

#include "iq8lane.cuh"

using namespace cbmoe;

template <int T>
static int run(const uint8_t* blocks, const float* table, float* out) {
  constexpr int BB = IqFmt<T>::kBytes;
  uint32_t words[32][Iq8Fmt<T>::kLaneWords];
  for (int lane = 0; lane < 32; ++lane) {
    const int g = lane >> 2;
    if (!iq8_lane_words<T>(blocks + g * BB, blocks + (g + 8) * BB, table, lane, words[lane])) return 1;
  }
  auto put = [&](int row, int p, uint32_t byte) {
    const int v = T == CBMOE_GGML_IQ2_S ? (int)(int8_t)(uint8_t)byte : 2 * (int)byte - 15;
    const uint8_t* blk = blocks + row * BB;
    const int m = T == CBMOE_GGML_IQ2_S ? p / 16 : p / 32;
    out[row * 256 + p] = (float)(v * (int)iq8_group_factor<T>(blk, m)) * iq8_block_scale<T>(blk);
  };
  for (int lane = 0; lane < 32; ++lane) {
    const int g = lane >> 2, t = lane & 3;
    for (int c = 0; c < 4; ++c) {
      if constexpr (T == CBMOE_GGML_IQ2_S) {
        uint32_t ag[4], ah[4];
        iq8_frag_iq2(words[lane][3 * c], words[lane][3 * c + 1], words[lane][3 * c + 2], ag, ah);
        for (int j = 0; j < 4; ++j)
          for (int b = 0; b < 4; ++b) {
            const int p = 64 * c + 16 * j + 4 * t + b;   // k = 4t + b of k16 step j (group 4c + j)
            if (iq8_perm<T>(16 * t + 4 * j + b) != p - 64 * c) return 2;   // B byte of the same k
            put(g, p, (ag[j] >> (8 * b)) & 255u);
            put(g + 8, p, (ah[j] >> (8 * b)) & 255u);
          }
      } else {
        for (int h = 0; h < 2; ++h) {
          uint32_t a[4];
          iq8_frag_iq3(words[lane][4 * c + 2 * h], words[lane][4 * c + 2 * h + 1], a);
          for (int b = 0; b < 4; ++b) {
            const int p0 = 64 * c + 32 * h + 4 * t + b, p1 = p0 + 16;   // k = 4t + b and 16 + 4t + b of step h
            if (iq8_perm<T>(16 * t + 8 * h + b) != p0 - 64 * c) return 2;
            if (iq8_perm<T>(16 * t + 8 * h + 4 + b) != p1 - 64 * c) return 2;
            put(g, p0, (a[0] >> (8 * b)) & 255u);
            put(g + 8, p0, (a[1] >> (8 * b)) & 255u);
            put(g, p1, (a[2] >> (8 * b)) & 255u);
            put(g + 8, p1, (a[3] >> (8 * b)) & 255u);
          }
        }
      }
    }
  }
  return 0;
}

// blocks: 16 raw blocks (row r's block at r * block bytes); out: [16][256] fp32.
extern "C" int iq8_host_reconstruct(int type, const uint8_t* blocks, const float* table, float* out) {
  switch (type) {
    case CBMOE_GGML_IQ2_S: return run<CBMOE_GGML_IQ2_S>(blocks, table, out);
    case CBMOE_GGML_IQ3_S: return run<CBMOE_GGML_IQ3_S>(blocks, table, out);
    default: return -1;
  }
}
