// TMA tensor maps: Q8_0 weight rows viewed as [rows][row_bytes / 8] 8-byte
// elements (one copy lands a box of rows as dense shared-memory rows of the
// box width; rows and columns past the matrix read as zeros), and fp16
// activation rows with the 64-byte swizzle of the tcgen05 operand layout.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace lfm3 {

// Encodes a map over Q8_0 rows viewed as [rows][row_bytes / 8] 8-byte
// elements (row_bytes a multiple of 16), boxes of box_bytes (a multiple of
// 16, <= 2048) x box_rows: one copy lands box_rows dense rows of box_bytes.
cudaError_t encode_q8_rows(CUtensorMap* map, const void* base, size_t row_bytes,
                           int rows, int box_bytes, int box_rows);

// Encodes a map over fp16 activations [rows][cols] (row pitch cols * 2
// bytes) with boxes of box_rows x box_cols (box_cols * 2 == 64) and the
// 64-byte swizzle the tcgen05 K-major operand layout expects.
cudaError_t encode_activation_map(CUtensorMap* map, const void* base, int rows,
                                  int cols, int box_rows, int box_cols);

// The same maps from a process-wide cache keyed by every encode argument
// (a hit is exactly the map the encoder would write).
cudaError_t cached_q8_rows(CUtensorMap* map, const void* base, size_t row_bytes,
                           int rows, int box_bytes, int box_rows);
cudaError_t cached_activation_map(CUtensorMap* map, const void* base, int rows,
                                  int cols, int box_rows, int box_cols);

}  // namespace lfm3
