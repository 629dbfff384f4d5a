// thunderfft_layout_tuned.h — shared-memory layouts for device-API callers.
//
// bench_layout<T, N, BPB>::L_in / L_out name the layouts the reference's
// validation and benchmark kernels stage tiles in
// (reference: include/thunderfft/thunderfft_layout_tuned.h:6-98).  This
// library's helpers accept any layout_t; these are its own choice: one
// padding element every 32 (bank-conflict-free strided staging), which fits
// the (N + pad_h(N)) * BPB workspace of the standard launch.
#pragma once

#include "thunderfft.cuh"

namespace thunderfft {

template <typename T, int N, int BPB>
struct bench_layout {
  static_assert(std::is_same_v<T, float> || std::is_same_v<T, half>, "float and half only");
  using L_in = layout_t<N, BPB, 1, N, 32, 1, false>;
  using L_out = layout_t<N, BPB, 1, N, 32, 1, false>;
};

}  // namespace thunderfft
