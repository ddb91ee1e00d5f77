// Primitive-op tensors of the tnn_* surface (inputs, uploads, downloads).
#pragma once
#include "session.cuh"

namespace tb2 {

int prim_upload_f64(Session* s, Tensor* t, const double* data, size_t n);
int prim_upload_i64(Session* s, Tensor* t, const long* data, size_t n);
int prim_download_f64(Session* s, Tensor* t, double* dst, size_t n);

}  // namespace tb2
