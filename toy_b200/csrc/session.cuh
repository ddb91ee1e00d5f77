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
class KvEngine;

// The decode engine of a session (kv.cu), freed before the step engine whose weights it reads.
void kv_free(Session* s);

// Data-parallel gradient reduction (dp.cu).
void dp_free(Session* s);
int nccl_allreduce_entry(void* ctx, float* buf, long long n, cudaStream_t st);
// 0, or the code that ended the session's communicator
int dp_status(const Session* s);
// Wait (host, bounded, next to the communicator's error state) for the step
// stream of a data-parallel session; 0 when it is idle.
int dp_wait_step(Session* s);

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
  Tensor* src[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  double fp[12] = {0};
  int ip[4] = {0};
  bool persistent = false;
  bool is_param = false;
  bool is_output = false;
  Tensor* view_of = nullptr;
  // primitive graph extras
  size_t view_off = 0;       // aliasing view: byte offset into view_of's buffer
  Tensor* grad = nullptr;    // autograd: the node holding d loss / d this
  bool is_loss = false;
  void* q8v = nullptr;       // Q8_0 tensor: int8 quants [rows][ne0]
  void* q8s = nullptr;       //              fp16 scale bits [rows][ne0 / 32]
  void* planes = nullptr;    // split-bf16 copy of a GEMM operand (hi then lo)
  void* outpad = nullptr;    // GEMM result with its rows padded to 4 floats (when ne0 % 4)
  long long nel() const { return (long long)ne[0] * ne[1] * ne[2] * ne[3]; }
  long long rows() const { return (long long)ne[1] * ne[2] * ne[3]; }
};

struct Session {
  int kind = 1;
  int device = 0;
  std::unique_ptr<LlamaEngine> eng;
  std::vector<std::unique_ptr<Tensor>> tensors;
  Tensor* io[TB2_IO_COUNT] = {nullptr};
  bool first_pending = false;
  DpState* dp = nullptr;
  KvEngine* kv = nullptr;
  // primitive op graph
  std::vector<Tensor*> nodes;     // forward program (topological order)
  std::vector<Tensor*> bwd;       // backward program (creation order)
  std::vector<Tensor*> ext;       // appended nodes (optimizer steps)
  std::vector<Tensor*> roots;     // extra forward roots (tnn_add_to_graph / outputs)
  Tensor* loss = nullptr;
  Tensor* ones = nullptr;         // d loss / d loss
  bool prim_realized = false;
  bool bwd_built = false;
  bool reset_pending = false;     // zero optimizer moments at the next backward
  cudaStream_t pstream = nullptr;
  // tnn_scratch_* host staging (16 MiB of f32) and the attached weight region
  std::vector<float> scratch;
  const uint8_t* mmap_base = nullptr;
  size_t mmap_size = 0;
  ~Session();
};

}  // namespace tb2
