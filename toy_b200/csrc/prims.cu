// Primitive-op tensors: device buffers created through tnn_input_* and
// filled / read through the tnn_* I/O calls (f64 <-> f32, i64 -> i32 narrowing
// as tinynn_ggml.c's upload_from_float_array / upload_from_int_array do).
#include <cstring>
#include <vector>

#include "prims.cuh"

namespace tb2 {

Session::~Session() {
  if (device >= 0) cudaSetDevice(device);
  dp_free(this);
  for (auto& t : tensors)
    if (t->data && !t->view_of) cudaFree(t->data);
  if (pstream) cudaStreamDestroy(pstream);
}

namespace {

int ensure_data(Tensor* t) {
  if (t->data) return 0;
  const size_t elem = t->type == 26 ? 4 : 4;
  t->bytes = (size_t)t->nel() * elem;
  if (cudaMalloc(&t->data, t->bytes ? t->bytes : 4) != cudaSuccess) {
    t->data = nullptr;
    return -3;
  }
  return cudaMemset(t->data, 0, t->bytes ? t->bytes : 4) == cudaSuccess ? 0 : -3;
}

}  // namespace

int prim_upload_f64(Session* s, Tensor* t, const double* data, size_t n) {
  (void)s;
  if (t->type != 0 || (long long)n > t->nel()) return -2;
  if (ensure_data(t)) return -3;
  std::vector<float> h(n);
  for (size_t i = 0; i < n; ++i) h[i] = (float)data[i];
  return cudaMemcpy(t->data, h.data(), n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -3;
}

int prim_upload_i64(Session* s, Tensor* t, const long* data, size_t n) {
  (void)s;
  if (t->type != 26 || (long long)n > t->nel()) return -2;
  if (ensure_data(t)) return -3;
  std::vector<int> h(n);
  for (size_t i = 0; i < n; ++i) h[i] = (int)data[i];
  return cudaMemcpy(t->data, h.data(), n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -3;
}

int prim_download_f64(Session* s, Tensor* t, double* dst, size_t n) {
  (void)s;
  if ((long long)n > t->nel()) return -2;
  if (!t->data) return -2;
  if (cudaDeviceSynchronize() != cudaSuccess) return -3;
  if (t->type == 26) {
    std::vector<int> h(n);
    if (cudaMemcpy(h.data(), t->data, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -3;
    for (size_t i = 0; i < n; ++i) dst[i] = h[i];
    return 0;
  }
  std::vector<float> h(n);
  if (cudaMemcpy(h.data(), t->data, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -3;
  for (size_t i = 0; i < n; ++i) dst[i] = h[i];
  return 0;
}

}  // namespace tb2
