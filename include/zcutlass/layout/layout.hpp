// Matrix layout tags.
//
// Same enum and helpers as the reference (include/zcutlass/layout/layout.hpp:5-31
// in supercatking/zcutlass): GemmDesc carries LayoutKind values by position.
#pragma once

#include <cstdint>

namespace zcutlass::layout {

struct RowMajor {};
struct ColumnMajor {};

enum class LayoutKind {
  RowMajor,
  ColumnMajor,
};

struct MatrixLayout {
  LayoutKind kind = LayoutKind::RowMajor;
  int64_t stride = 0;
};

// Element offset of (row, col) in a matrix with the given layout and leading
// dimension.
inline int64_t offset(MatrixLayout layout, int64_t row, int64_t col) {
  return layout.kind == LayoutKind::RowMajor ? row * layout.stride + col
                                             : col * layout.stride + row;
}

inline const char* layout_name(LayoutKind kind) {
  return kind == LayoutKind::RowMajor ? "row" : "column";
}

}  // namespace zcutlass::layout
