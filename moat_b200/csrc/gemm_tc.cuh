// Tensor-core (tcgen05) path of the INT4 super-block GEMM; see gemm_tc.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mb {
namespace tc {

struct TcPlan {
  bool ok = false;
  int NP = 0;       // MMA N: batch padded to 16 or 32
  int Ck = 1;       // CTAs per cluster (K split)
  int S = 0;        // stage ring depth
  int ctas = 0;
  int xoff = 0, xblocks = 0, baroff = 0;
  int smem = 0;     // dynamic shared memory bytes
  int tcols = 0;    // TMEM columns per CTA
};

// Plans the launch for one block of up to 32 batch rows; false if the shape is not
// supported by this path (M % 256 != 0, K % 8 != 0, or a K slice too long).
bool plan(int N, int K, int M, int sms, TcPlan* pl);

int launch(const TcPlan& pl, const uint16_t* act, const uint8_t* sb, uint16_t* out, int N, int K, int M,
           uint32_t* err, cudaStream_t st);

}  // namespace tc
}  // namespace mb
