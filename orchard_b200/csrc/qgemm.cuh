// Arguments of the quantised skinny-GEMM kernel family (qgemm.cu).
#pragma once

#include "orch_common.cuh"

namespace orch {

enum { W_Q4 = 0, W_Q8G = 1, W_Q8PC = 2 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

struct QArgs {
  const uint8_t* w;   // packed weights [N, K/2] (INT4) or [N, K] (INT8)
  const __half* s;    // scales [N, K/32] or [N] (per channel)
  const void* x;      // activations [M, K], fp16 or fp32
  int x_f32;
  int M, N, K;
  int nchunk;         // ceil(K / 128), set by the launcher
  // STORE / RESID / SWIGLU / QKV(q) output
  void* out;
  int out_f32;
  int ldo;
  // QKV + RoPE + KV append
  int H, nh, hd, max_seq, max_pos;
  const int* pos;
  const int* slots;
  const float* cos_tab;
  const float* sin_tab;
  __half* kc;
  __half* vc;
  const float* lora_t;
  const float* lora_b;
  int lora_r;
  uint32_t* check;
};

template <int WF, int EPI>
int qgemm_run(QArgs a, cudaStream_t st);

}  // namespace orch
