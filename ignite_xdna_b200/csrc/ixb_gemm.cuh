// int8 GEMM + pow2 SRS and W4A8 GEMM/GEMV entry points.
#pragma once
#include "../../include/ixb200.h"

extern "C" {
int ixb_i8gemm_srs(const int8_t*, const int8_t*, const int32_t*, int8_t*, int, int, int, int, void*) {
  return IXB_ERR_UNSUPPORTED;
}
int ixb_i8gemm_i32(const int8_t*, const int8_t*, int32_t*, int, int, int, void*) { return IXB_ERR_UNSUPPORTED; }
int ixb_w4a8_gemm(const int8_t*, const uint8_t*, const int8_t*, const int32_t*, int8_t*, int, int, int, void*) {
  return IXB_ERR_UNSUPPORTED;
}
int ixb_w4a8_gemv(const int8_t*, const uint8_t*, const int8_t*, const int32_t*, int8_t*, int, int, void*) {
  return IXB_ERR_UNSUPPORTED;
}
}
