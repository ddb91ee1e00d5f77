// Session and tensor handles behind the opaque void* of the C ABI.
#pragma once
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "engine.cuh"
#include "toy_b200.h"

namespace tb2 {

struct Session;
struct DpState;

// Data-parallel gradient reduction (dp.cu).
void dp_free(Session* s);
int nccl_allreduce_entry(void* ctx, float* buf, long long n, cudaStream_t st);

struct Tensor {
  enum Role : int { kPrim = 0, kIds, kPos, kLabels, kHp, kLoss, kParam };
  Session* sess = nullptr;
  int role = kPrim;
  int ne[4] = {1, 1, 1, 1};
  int type = 0;             // ggml type ids: 0 f32, 8 q8_0, 26 i32
  std::string name;
  std::string param;        // engine parameter name (role kParam)
  // primitive graph node (role kPrim)
  void* data = nullptr;     // device buffer (owned unless view_of is set)
  size_t bytes = 0;
  int op = 0;               // 0 = leaf
  Tensor* src[4] = {nullptr, nullptr, nullptr, nullptr};
  double fp[12] = {0};
  int ip[4] = {0};
  bool persistent = false;
  bool is_param = false;
  bool is_output = false;
  Tensor* view_of = nullptr;
  long long nel() const { return (long long)ne[0] * ne[1] * ne[2] * ne[3]; }
};

struct Session {
  int kind = 1;
  int device = 0;
  std::unique_ptr<LlamaEngine> eng;
  std::vector<std::unique_ptr<Tensor>> tensors;
  Tensor* io[TB2_IO_COUNT] = {nullptr};
  bool first_pending = false;
  DpState* dp = nullptr;
  // primitive op graph
  std::vector<Tensor*> nodes;
  bool prim_realized = false;
  cudaStream_t pstream = nullptr;
  ~Session();
};

}  // namespace tb2
