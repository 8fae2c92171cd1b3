// repack.cpp: the reference's weight bytes (palette.Linear, shiftScale's offset form, MXFP4) into
// the integer-MMA tiles of common.h (tile_pos gives every code's place). Every code is copied as it is, so the dequantisation of the
// tiles equals the format's own (checked by hc_linear_dequant).
#include "repack.h"

#include <algorithm>
#include <cstring>
#include <string>
#include <thread>

namespace hc {

std::vector<RowRef> rows_of(const hc_linear_desc &d) {
  std::vector<RowRef> v(d.rows);
  for (uint32_t r = 0; r < d.rows; ++r) v[r] = {&d, r};
  return v;
}

std::vector<RowRef> rows_concat(const std::vector<const hc_linear_desc *> &ds) {
  std::vector<RowRef> v;
  for (auto *d : ds)
    for (uint32_t r = 0; r < d->rows; ++r) v.push_back({d, r});
  return v;
}

std::vector<RowRef> rows_glu(const hc_linear_desc &gate, uint32_t gate_row0, uint32_t gate_step,
                             const hc_linear_desc &up, uint32_t up_row0, uint32_t up_step,
                             uint32_t n) {
  constexpr uint32_t half = kTileRows / 2;
  std::vector<RowRef> v;
  for (uint32_t t = 0; t < (n + half - 1) / half; ++t) {
    for (uint32_t j = 0; j < half; ++j) {
      uint32_t o = t * half + j;
      v.push_back(o < n ? RowRef{&gate, gate_row0 + o * gate_step} : RowRef{nullptr, 0});
    }
    for (uint32_t j = 0; j < half; ++j) {
      uint32_t o = t * half + j;
      v.push_back(o < n ? RowRef{&up, up_row0 + o * up_step} : RowRef{nullptr, 0});
    }
  }
  return v;
}

namespace {

// The code of (row, col) as the kernels read it: int8 as its byte; int4 unsigned 0..15 (the
// symmetric format's two's complement nibble n as n ^ 8 = q + 8); MXFP4 its e2m1 nibble.
inline uint8_t code_of(const RowRef &rr, uint32_t col) {
  const hc_linear_desc *d = rr.d;
  if (!d || col >= d->cols) return 0;
  const uint8_t *p = static_cast<const uint8_t *>(d->data);
  const size_t i = size_t(rr.row) * d->cols + col;
  switch (d->format) {
    case HC_FMT_INT8_ROW: return p[i];
    case HC_FMT_INT4_SYM_G32: return uint8_t(((p[i / 2] >> (4 * (i % 2))) & 0xf) ^ 8);
    default: return uint8_t((p[i / 2] >> (4 * (i % 2))) & 0xf);
  }
}

// fp16 scale / zero of (row, group) for the int4 formats; zeros of padding.
inline void sz_of(const RowRef &rr, uint32_t grp, uint16_t *s, uint16_t *z) {
  const hc_linear_desc *d = rr.d;
  if (!d || grp >= d->cols / 32) { *s = 0; *z = 0; return; }
  const size_t j = size_t(rr.row) * (d->cols / 32) + grp;
  *s = d->scales[j];
  *z = d->format == HC_FMT_INT4_SYM_G32 ? uint16_t(0x4800) /* 8.0 */ : d->zeros[j];
}

inline uint8_t e_of(const RowRef &rr, uint32_t grp) {
  const hc_linear_desc *d = rr.d;
  if (!d || grp >= d->cols / 32) return 0;
  return d->exps[size_t(rr.row) * (d->cols / 32) + grp];
}

}  // namespace

char *repack(const std::vector<RowRef> &rows, Packed *out) {
  const hc_linear_desc *first = nullptr;
  for (auto &r : rows)
    if (r.d) { first = r.d; break; }
  if (!first) return make_error("repack: no rows");
  for (auto &r : rows) {
    if (!r.d) continue;
    if (r.d->format != first->format || r.d->cols != first->cols)
      return make_error("repack: fused matrices differ in format or columns");
    if (!r.d->data) return make_error("repack: matrix without data");
    if (r.row >= r.d->rows) return make_error("repack: row out of range");
  }
  Packed &P = *out;
  P.fmt = first->format;
  switch (first->format) {
    case HC_FMT_INT8_ROW: P.kind = kKindInt8; P.tile_bytes = kTileInt8; break;
    case HC_FMT_INT4_SYM_G32:
    case HC_FMT_INT4_ASYM_G32: P.kind = kKindInt4; P.tile_bytes = kTileInt4; break;
    case HC_FMT_MXFP4: P.kind = kKindMx; P.tile_bytes = kTileMx; break;
    default: return make_error("repack: format " + std::to_string(first->format) + " has no integer tiles");
  }
  if (P.kind != kKindInt8 && first->cols % 32)
    return make_error("repack: columns not a multiple of 32");
  for (auto &r : rows) {
    if (!r.d) continue;
    if (P.kind == kKindInt8 && !r.d->scales) return make_error("repack: int8 without scales");
    if (P.kind == kKindInt4 && !r.d->scales) return make_error("repack: int4 without scales");
    if (r.d->format == HC_FMT_INT4_ASYM_G32 && !r.d->zeros) return make_error("repack: int4 asym without zeros");
    if (P.kind == kKindMx && !r.d->exps) return make_error("repack: MXFP4 without exponents");
  }
  P.rows = int(rows.size());
  P.cols = int(first->cols);
  P.rows_p = pad_to(P.rows, kTileRows);
  P.cols_p = pad_to(P.cols, kTileCols);
  P.rtiles = P.rows_p / kTileRows;
  P.ktiles = P.cols_p / kTileCols;
  P.tiles.assign(size_t(P.rtiles) * P.ktiles * P.tile_bytes, 0);
  bool any_bias = false;
  for (auto &r : rows) any_bias |= r.d && r.d->bias;
  if (any_bias) {
    P.bias.assign(P.rows_p, 0.0f);
    for (size_t i = 0; i < rows.size(); ++i)
      if (rows[i].d && rows[i].d->bias) P.bias[i] = rows[i].d->bias[rows[i].row];
  }
  if (P.kind == kKindInt8) {
    P.row_scale.assign(P.rows_p, 0.0f);
    for (size_t i = 0; i < rows.size(); ++i)
      if (rows[i].d) P.row_scale[i] = f16_value(rows[i].d->scales[rows[i].row]);
  }
  const int kind4 = P.kind != kKindInt8, mx = P.kind == kKindMx;
  auto work = [&](int rt0, int rt1) {
    RowRef pad{nullptr, 0};
    for (int rt = rt0; rt < rt1; ++rt) {
      const RowRef *rr[kTileRows];
      for (int r = 0; r < kTileRows; ++r) {
        size_t row = size_t(rt) * kTileRows + r;
        rr[r] = row < rows.size() ? &rows[row] : &pad;
      }
      for (int kt = 0; kt < P.ktiles; ++kt) {
        uint8_t *t = &P.tiles[(size_t(rt) * P.ktiles + kt) * P.tile_bytes];
        const uint32_t col0 = uint32_t(kt) * kTileCols;
        for (int r = 0; r < kTileRows; ++r)
          for (int cc = 0; cc < kTileCols; ++cc) {
            const TilePos tp = tile_pos(kind4, mx, r, cc);
            const uint8_t code = code_of(*rr[r], col0 + cc);
            t[tp.byte] = uint8_t(t[tp.byte] | (kind4 ? uint8_t((code & 0xf) << tp.shift) : code));
          }
        if (!kind4) continue;
        for (int r = 0; r < kTileRows; ++r)
          for (int G = 0; G < kGroupsPerTile; ++G) {
            const TilePos tp = tile_pos(kind4, mx, r, G * kGroup);
            const uint32_t grp = uint32_t(kt) * kGroupsPerTile + G;
            if (P.kind == kKindInt4) {
              uint16_t sv, zv;
              sz_of(*rr[r], grp, &sv, &zv);
              std::memcpy(t + kTileCodes4 + tp.lane * 16 + 2 * tp.sidx, &sv, 2);
              std::memcpy(t + kTileCodes4 + tp.lane * 16 + 8 + 2 * tp.sidx, &zv, 2);
            } else {
              t[kTileCodes4 + tp.lane * 4 + tp.sidx] = e_of(*rr[r], grp);
            }
          }
      }
    }
  };
  unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  int nt = int(std::min<unsigned>(hw, unsigned(P.rtiles)));
  std::vector<std::thread> th;
  int per = (P.rtiles + nt - 1) / nt;
  for (int i = 0; i < nt; ++i) {
    int lo = i * per, hi = std::min(P.rtiles, lo + per);
    if (lo < hi) th.emplace_back(work, lo, hi);
  }
  for (auto &x : th) x.join();
  return nullptr;
}

}  // namespace hc
