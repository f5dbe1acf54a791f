// Implicit-GEMM 2-D convolution (conv.cu): NHWC input, weights [O][KH][KW][C].
#pragma once

#include <cuda_runtime.h>

#include "gemm.h"

namespace es {

struct ConvArgs {
  const void* x = nullptr;     // [B][Hin][Win][C]
  const void* w = nullptr;     // [O][KH][KW][C]
  const float* bias = nullptr; // [O] or null
  void* out = nullptr;         // [B][Hout][Wout][O], Hout = Hin + ph + ph_hi - KH + 1
  int dtype = kDtypeBF16;      // x, w and out share it
  int B = 0, Hin = 0, Win = 0, C = 0, O = 0, KH = 0, KW = 0;
  int ph = 0, pw = 0;          // zero padding before the first row / column
  int ph_hi = -1, pw_hi = -1;  // zero padding after the last (-1: the same as before)
  int* err = nullptr;
  int num_sms = 148;
  int persistent = 1;          // 1 persistent CTAs (default), 0 one tile per CTA (tuning)
  int kernel = 0;              // 0 auto (the pair kernel with resident weights where it fits), 1 conv.cu's kernel
  unsigned long long* prof = nullptr;  // pair kernel: wait-cycle counters (tuning), null when off
  // ghost rows (pair kernel only): the input continues gtop rows above and
  // gbot rows below x in ghosts [B][gtop + gbot][Win][C]; the zero padding
  // ph / ph_hi lies beyond them
  const void* ghosts = nullptr;
  int gtop = 0, gbot = 0;
  int ghost_wpitch = 0, ghost_w0 = 0;  // ghost rows of ghost_wpitch pixels (0: Win), x's columns from ghost_w0
  // output rows of out_wpitch pixels (0: Wout), the computed columns written from
  // column out_w0 on (pair kernel only): a conv that fills a column range of out
  int out_wpitch = 0, out_w0 = 0;
};

inline int conv_ghost_rows(const ConvArgs& a) { return a.gtop + a.gbot; }
template <class Args>
inline int conv_ghost_rows(const Args&) { return 0; }

template <class Args>
inline int conv_hout(const Args& a) {
  return a.Hin + conv_ghost_rows(a) + a.ph + (a.ph_hi < 0 ? a.ph : a.ph_hi) - a.KH + 1;
}
template <class Args>
inline int conv_wout(const Args& a) {
  return a.Win + a.pw + (a.pw_hi < 0 ? a.pw : a.pw_hi) - a.KW + 1;
}

const char* check_conv_args(const ConvArgs& a);
int conv_launch(const ConvArgs& a, cudaStream_t stream);
// The CTA-pair kernel with the weights resident in shared memory (conv_pair.cu).
bool conv_pair_eligible(const ConvArgs& a);
// Output-channel tile the pair kernel would use for this shape (0: it does not
// take the shape: channel counts or a weight slice too large for shared memory).
int conv_pair_otile(int C, int O, int KH, int KW);
int conv_pair_launch(const ConvArgs& a, cudaStream_t stream);

// Weight gradient of conv_launch's convolution: dw[o][kh][kw][c] (fp32, must be
// zero on entry) += sum over output pixels of dy[b][h][w][o] * x[b][h+kh-ph][w+kw-pw][c].
struct ConvWgradArgs {
  const void* x = nullptr;     // [B][Hin][Win][C]
  const void* dy = nullptr;    // [B][Hout][Wout][O]
  float* dw = nullptr;         // [O][KH][KW][C] fp32
  int dtype = kDtypeBF16;      // x and dy share it
  int B = 0, Hin = 0, Win = 0, C = 0, O = 0, KH = 0, KW = 0;
  int ph = 0, pw = 0;
  int ph_hi = -1, pw_hi = -1;
  int* err = nullptr;
  int num_sms = 148;
};

const char* check_conv_wgrad_args(const ConvWgradArgs& a);
int conv_wgrad_launch(const ConvWgradArgs& a, cudaStream_t stream);

}  // namespace es
