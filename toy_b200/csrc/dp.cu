// Data parallelism: every rank holds a full replica and its own batch; after
// the backward the trainable-gradient arena (one contiguous f32 buffer) is
// summed across ranks with NCCL on the step stream, and AdamW applies the
// 1/world scale. The all-reduce is enqueued inside the step program, so it is
// captured in the step's CUDA graph like every other launch.
#include <nccl.h>

#include <cstring>

#include "session.cuh"
#include "toy_b200.h"

namespace tb2 {

struct DpState {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
};

namespace {

int nccl_allreduce(void* ctx, float* buf, long long n, cudaStream_t st) {
  DpState* d = static_cast<DpState*>(ctx);
  if (!d || !d->comm) return -2;
  return ncclAllReduce(buf, buf, (size_t)n, ncclFloat32, ncclSum, d->comm, st) == ncclSuccess ? 0 : -3;
}

}  // namespace

int nccl_allreduce_entry(void* ctx, float* buf, long long n, cudaStream_t st) { return nccl_allreduce(ctx, buf, n, st); }

void dp_free(Session* s) {
  if (!s || !s->dp) return;
  if (s->eng) {
    s->eng->drop_graph();   // a graph holding NCCL work must go before its communicator
    s->eng->set_allreduce_hook(nullptr, nullptr);
    s->eng->set_grad_scale(1.0f);
  }
  if (s->dp->comm) ncclCommDestroy(s->dp->comm);
  delete s->dp;
  s->dp = nullptr;
}

}  // namespace tb2

using tb2::DpState;
using tb2::Session;

extern "C" {

int tb2_nccl_unique_id(void* out, size_t nbytes) {
  if (!out || nbytes < sizeof(ncclUniqueId)) return -1;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return -3;
  std::memcpy(out, &id, sizeof(id));
  return (int)sizeof(id);
}

int tb2_dp_init(void* sess, const void* unique_id, int rank, int world) {
  if (!sess || !unique_id || world < 1 || rank < 0 || rank >= world) return -1;
  Session* s = static_cast<Session*>(sess);
  if (!s->eng || s->dp) return -2;
  if (cudaSetDevice(s->device) != cudaSuccess) return -3;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  auto* d = new DpState();
  d->rank = rank;
  d->world = world;
  if (ncclCommInitRank(&d->comm, world, id, rank) != ncclSuccess) {
    delete d;
    return -3;
  }
  s->dp = d;
  s->eng->set_allreduce_hook(tb2::nccl_allreduce_entry, d);
  s->eng->set_grad_scale(1.0f / (float)world);
  return 0;
}

int tb2_dp_set_bucket_floats(void* sess, long long floats) {
  if (!sess || floats < 1) return -1;
  Session* s = static_cast<Session*>(sess);
  if (!s->eng) return -2;
  s->eng->set_bucket_floats(floats);
  return 0;
}

int tb2_dp_free(void* sess) {
  if (!sess) return -1;
  tb2::dp_free(static_cast<Session*>(sess));
  return 0;
}

}  // extern "C"
