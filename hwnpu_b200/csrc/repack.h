// repack.h: host repacking of the reference's weight layouts into the kernels' tiles.
#ifndef HWNPU_REPACK_H
#define HWNPU_REPACK_H

#include <vector>

#include "common.h"

namespace hc {

uint16_t f16_bits(float f);
float f16_value(uint16_t h);

// One output row of a (possibly fused) matrix: row `row` of the matrix `d`; d == nullptr is a
// padding row of zeros.
struct RowRef {
  const hc_linear_desc *d;
  uint32_t row;
};

// A matrix in tiles of kTileRows x kTileCols: tiles [rtiles][ktiles][tile_bytes] (see
// common.h for the layout inside a tile), float row scales for kKindInt8, float biases.
struct Packed {
  Kind kind = kKindInt8;
  int fmt = HC_FMT_NONE;  // the source format
  int rows = 0, cols = 0, rows_p = 0, cols_p = 0, rtiles = 0, ktiles = 0, tile_bytes = 0;
  std::vector<uint8_t> tiles;
  std::vector<float> row_scale;
  std::vector<float> bias;
};

std::vector<RowRef> rows_of(const hc_linear_desc &d);
// q rows, then k rows, then v rows (one fused projection).
std::vector<RowRef> rows_concat(const std::vector<const hc_linear_desc *> &ds);
// Tiles of 8 gate rows then the 8 up rows of the same outputs, for the SwiGLU epilogue:
// gate row j comes from (gate, gate_row0 + j * gate_step), up row j from (up, up_row0 + j * up_step).
std::vector<RowRef> rows_glu(const hc_linear_desc &gate, uint32_t gate_row0, uint32_t gate_step,
                             const hc_linear_desc &up, uint32_t up_row0, uint32_t up_step,
                             uint32_t n);

// Checks the sources (one format, equal columns) and writes the tiles; NULL or an error.
char *repack(const std::vector<RowRef> &rows, Packed *out);

}  // namespace hc

#endif
