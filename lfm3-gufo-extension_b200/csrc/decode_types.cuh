// Device-side descriptions shared by the decode kernels.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace lfm3 {

constexpr int kMaxBatch = 8;  // engine.hpp:48 (Session::kMaxBatch)

// One layer's recurrent state of one session, in the reference's layout
// (engine.cpp:55-77): convolution history f32[hidden][width - 1]
// channel-major, or separate F16 K and V rings [capacity][kv_heads][128]
// with row t in slot t % capacity.
struct LayerState {
  float* conv;
  __half* k;
  __half* v;
  int capacity;
  int pad;
};

// The rows of one decode round: row r belongs to a session at `position`
// whose per-layer states are layers[r][0..n_layers).
struct DecodeRows {
  int count;
  int pad;
  int position[kMaxBatch];
  uint32_t token[kMaxBatch];
  const LayerState* layers[kMaxBatch];
};

}  // namespace lfm3
