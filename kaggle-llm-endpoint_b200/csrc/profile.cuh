// Kernel kinds for launch accounting and per-kernel event timing (profile.cu, cbmoe_profile_read).
#pragma once
#include <cuda_runtime.h>

#include "cbmoe.h"

namespace cbmoe {

enum ProfKind {
  kProfPlan = 0,          // route_plan_kernel
  kProfCb3GateUp = 1,     // decode_kernel_t<CB3, 2 matrices, SWIGLU>
  kProfCb3Down = 2,       // decode_kernel_t<CB3, 1 matrix, STORE, hi/lo B>
  kProfCb3Single = 3,     // decode_kernel_t<CB3, 1 matrix, STORE>
  kProfW8GateUp = 4,      // decode_kernel_t<W8, 2 matrices, SWIGLU>
  kProfW8Down = 5,        // decode_kernel_t<W8, 1 matrix, STORE, hi/lo B>
  kProfW8Single = 6,      // decode_kernel_t<W8, 1 matrix, STORE>
  kProfCombine = 7,       // combine_kernel
  kProfOther = 8,         // layout repacks, dequant checks, row gathers
  kProfGrpCb3GateUp = 9,  // grouped_kernel<CB3, gate+up, SWIGLU> (tcgen05)
  kProfGrpCb3Down = 10,   // grouped_kernel<CB3, down, STORE>
  kProfGrpW8GateUp = 11,  // grouped_kernel<W8, gate+up, SWIGLU>
  kProfGrpW8Store = 12,   // grouped_kernel<W8, one matrix, STORE>
  kProfExchange = 13,     // expert-parallel NCCL dispatch or return (one send/recv group)
  kProfIqGateUp = 14,     // iq_matvec_kernel over gate or up (raw GGUF IQ tables), and the SwiGLU between
  kProfIqDown = 15,       // iq_matvec_kernel over down
  kProfKinds = 16
};

void prof_begin(int kind, cudaStream_t s);
void prof_end(int kind, cudaStream_t s);
// Launches counted besides the one prof_begin counts (a kind timed as one span over several kernels).
void prof_add_launches(int n);

}  // namespace cbmoe
