// TMA tensor maps over Q8_0 weight rows: the bytes of a matrix viewed as a
// 3-D tensor [rows][row_bytes / 16][16], so one tiled copy moves a box of
// up to 256 rows x (17 x 16) bytes (one 256-column chunk of each row) into
// shared memory as dense 272-byte rows. Rows past the matrix read as zeros.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace lfm3 {

// Encodes a map over `rows` rows of `row_bytes` bytes (a multiple of 16)
// starting at base (16-byte aligned), with boxes of box_rows rows and
// chunk_bytes (a multiple of 16, <= 4096) per row. Returns cudaSuccess or the
// error of the driver call.
cudaError_t encode_row_map(CUtensorMap* map, const void* base,
                           size_t row_bytes, int rows, int chunk_bytes,
                           int box_rows);

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
