// Data parallelism: every rank holds a full replica and its own batch; the
// trainable-gradient arena (one contiguous f32 buffer) is summed across ranks
// with NCCL in buckets on a side stream while the backward runs (engine.cu
// bucket_ready), and AdamW applies the 1/world scale. The all-reduces are
// enqueued inside the step program, so they are captured in the step's CUDA
// graph like every other launch.
//
// Failure handling is host-side and never faults a GPU: the communicator is
// created non-blocking (ncclCommInitRankConfig, blocking = 0), and every host
// wait that can depend on a peer -- communicator creation, the enqueue of a
// collective, the end of a step -- polls ncclCommGetAsyncError next to the
// thing it waits for, with a time limit. An asynchronous NCCL error or the
// limit aborts the communicator (ncclCommAbort ends the collectives still
// running on the device), marks the session's data parallelism as failed and
// returns the code to the caller: -3 NCCL error, -4 time limit. A failed
// session refuses further steps (-2) until tb2_dp_free.
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <memory>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "session.cuh"
#include "toy_b200.h"

namespace tb2 {

struct DpState {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  int failed = 0;   // 0 healthy, else the code that ended the communicator
  Session* s = nullptr;
};

namespace {

long long g_timeout_ms = 120000;   // host limit on any wait that depends on a peer

// ncclCommAbort ends this rank's collectives and frees the communicator; it
// runs on a helper thread that the caller waits for within the time limit, so
// an abort that does not return (a peer gone mid-teardown) cannot hold the
// host: the communicator is then left to the helper and the process.
void abort_comm(DpState* d, int code) {
  ncclComm_t c = d->comm;
  d->comm = nullptr;
  if (!d->failed) d->failed = code;
  fprintf(stderr, "[toy_b200] data parallelism: rank %d of %d aborts its communicator (%s)\n", d->rank, d->world,
          code == -4 ? "time limit reached" : code == -6 ? "aborted by the caller" : "NCCL error");
  if (!c) return;
  auto done = std::make_shared<std::atomic<bool>>(false);
  std::thread([c, done]() {
    ncclCommAbort(c);
    done->store(true);
  }).detach();
  const auto t0 = std::chrono::steady_clock::now();
  while (!done->load()) {
    if (std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
        g_timeout_ms) {
      fprintf(stderr, "[toy_b200] data parallelism: rank %d: ncclCommAbort did not return within the limit\n",
              d->rank);
      return;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

// Poll ready() (> 0 done, 0 pending, < 0 error code) next to the
// communicator's asynchronous error, until done, an error, or the time limit.
template <class F>
int watch(DpState* d, F ready) {
  const auto t0 = std::chrono::steady_clock::now();
  for (long long it = 0;; ++it) {
    const int r = ready();
    if (r > 0) return 0;
    if (r < 0) return r;
    if (!d->comm) return d->failed ? d->failed : -2;
    ncclResult_t ae = ncclSuccess;
    if (ncclCommGetAsyncError(d->comm, &ae) != ncclSuccess || (ae != ncclSuccess && ae != ncclInProgress)) {
      abort_comm(d, -3);
      return -3;
    }
    const long long ms =
        std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms > g_timeout_ms) {
      abort_comm(d, -4);
      return -4;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(it < 200 ? 10 : 200));
  }
}

// A non-blocking communicator may answer ncclInProgress while an operation is
// still being set up; the next NCCL call may only follow once it is done.
int settle(DpState* d) {
  return watch(d, [d]() {
    ncclResult_t ae = ncclSuccess;
    if (ncclCommGetAsyncError(d->comm, &ae) != ncclSuccess) return -3;
    return ae == ncclInProgress ? 0 : 1;
  });
}

int nccl_allreduce(void* ctx, float* buf, long long n, cudaStream_t st) {
  DpState* d = static_cast<DpState*>(ctx);
  if (!d || !d->comm || d->failed) return -2;
  const ncclResult_t r = ncclAllReduce(buf, buf, (size_t)n, ncclFloat32, ncclSum, d->comm, st);
  if (r == ncclInProgress) return settle(d);
  return r == ncclSuccess ? 0 : -3;
}

// The end of a step (an event on the step stream, or the stream itself).
int wait_event(void* ctx, cudaEvent_t ev) {
  DpState* d = static_cast<DpState*>(ctx);
  return watch(d, [ev]() {
    const cudaError_t e = cudaEventQuery(ev);
    return e == cudaSuccess ? 1 : e == cudaErrorNotReady ? 0 : -3;
  });
}

}  // namespace

int nccl_allreduce_entry(void* ctx, float* buf, long long n, cudaStream_t st) { return nccl_allreduce(ctx, buf, n, st); }

int dp_status(const Session* s) { return s && s->dp ? s->dp->failed : 0; }

int dp_wait_step(Session* s) {
  if (!s || !s->dp || !s->eng) return 0;
  DpState* d = s->dp;
  if (d->failed) return d->failed;
  cudaStream_t st = s->eng->stream();
  return watch(d, [st]() {
    const cudaError_t e = cudaStreamQuery(st);
    return e == cudaSuccess ? 1 : e == cudaErrorNotReady ? 0 : -3;
  });
}

void dp_free(Session* s) {
  if (!s || !s->dp) return;
  if (s->eng) {
    s->eng->sync();
    s->eng->drop_graph();   // a graph holding NCCL work must go before its communicator
    s->eng->set_allreduce_hook(nullptr, nullptr);
    s->eng->set_wait_hook(nullptr, nullptr);
    s->eng->set_grad_scale(1.0f);
  }
  DpState* d = s->dp;
  if (d->comm) {
    // NCCL finalize + destroy: collective across the node's ranks, so every
    // rank frees together; a rank leaving alone aborts first (tb2_dp_abort).
    // A finalize that does not complete in time is left as it is (reported,
    // not aborted: an abort in the middle of a finalize is not bounded).
    const ncclResult_t r = ncclCommFinalize(d->comm);
    bool done = r == ncclSuccess;
    if (r == ncclInProgress) {
      const auto t0 = std::chrono::steady_clock::now();
      for (;;) {
        ncclResult_t ae = ncclSuccess;
        if (ncclCommGetAsyncError(d->comm, &ae) != ncclSuccess) break;
        if (ae != ncclInProgress) {
          done = ae == ncclSuccess;
          break;
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
            g_timeout_ms)
          break;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
      }
    }
    if (done) ncclCommDestroy(d->comm);
    else
      fprintf(stderr, "[toy_b200] data parallelism: rank %d: communicator finalize did not complete; left in place\n",
              d->rank);
    d->comm = nullptr;
  }
  delete d;
  s->dp = nullptr;
}

// The buckets the backward reduces, in issue order: the engine's own decision
// rule (LlamaEngine::bucket_take) replayed over the layers, last layer first,
// then the final flush of what is left (embedding, final norm).
long long bucket_plan(const long long* layer_lo, int n_layers, long long n_train, long long min_floats,
                      long long* out, long long cap) {
  long long pend_lo = n_train, pend_hi = n_train, n = 0, b_lo = 0, b_hi = 0;
  for (int l = n_layers - 1; l >= 0; --l) {
    if (LlamaEngine::bucket_take(pend_lo, pend_hi, layer_lo[l], false, min_floats, b_lo, b_hi)) {
      if (out && 2 * n + 1 < cap) {
        out[2 * n] = b_lo;
        out[2 * n + 1] = b_hi;
      }
      ++n;
    }
  }
  if (LlamaEngine::bucket_take(pend_lo, pend_hi, 0, true, min_floats, b_lo, b_hi)) {
    if (out && 2 * n + 1 < cap) {
      out[2 * n] = b_lo;
      out[2 * n + 1] = b_hi;
    }
    ++n;
  }
  return n;
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

int tb2_dp_set_timeout_ms(long long ms) {
  if (ms < 1) return -1;
  tb2::g_timeout_ms = ms;
  return 0;
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
  d->s = s;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const ncclResult_t r = ncclCommInitRankConfig(&d->comm, world, id, rank, &cfg);
  int rc = (r == ncclSuccess || r == ncclInProgress) && d->comm ? tb2::settle(d) : -3;
  if (rc) {
    if (d->comm) ncclCommAbort(d->comm);
    delete d;
    return rc;
  }
  s->dp = d;
  s->eng->set_allreduce_hook(tb2::nccl_allreduce_entry, d);
  s->eng->set_wait_hook(tb2::wait_event, d);
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

int tb2_dp_wait(void* sess) {
  if (!sess) return -1;
  return tb2::dp_wait_step(static_cast<Session*>(sess));
}

int tb2_dp_status(void* sess) {
  if (!sess) return -1;
  return tb2::dp_status(static_cast<Session*>(sess));
}

int tb2_dp_abort(void* sess) {
  if (!sess) return -1;
  Session* s = static_cast<Session*>(sess);
  if (!s->dp) return -2;
  tb2::abort_comm(s->dp, -6);
  return 0;
}

int tb2_dp_free(void* sess) {
  if (!sess) return -1;
  tb2::dp_free(static_cast<Session*>(sess));
  return 0;
}

long long tb2_dp_bucket_plan(const long long* layer_lo, int n_layers, long long n_train, long long bucket_floats,
                             long long* out, long long cap) {
  if ((!layer_lo && n_layers > 0) || n_layers < 0 || n_train < 0 || bucket_floats < 1 || cap < 0) return -1;
  for (int l = 0; l < n_layers; ++l)
    if (layer_lo[l] < 0 || layer_lo[l] > n_train || (l + 1 < n_layers && layer_lo[l] > layer_lo[l + 1])) return -1;
  return tb2::bucket_plan(layer_lo, n_layers, n_train, bucket_floats, out, cap);
}

long long tb2_dp_session_bucket_plan(void* sess, long long* out, long long cap) {
  if (!sess || cap < 0) return -1;
  Session* s = static_cast<Session*>(sess);
  if (!s->eng) return -2;
  const std::vector<long long> lo = s->eng->layer_grad_lo();
  return tb2::bucket_plan(lo.data(), (int)lo.size(), s->eng->n_trainable(), s->eng->bucket_floats(), out, cap);
}

}  // extern "C"
