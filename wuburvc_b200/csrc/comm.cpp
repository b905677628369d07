// comm.cpp — data-parallel gradient all-reduce over NCCL (loaded at run time).
//
// One process per GPU.  The flat gradient buffer is ordered by backward completion, so each
// stage of the backward finishes a contiguous range; that range is all-reduced on a separate
// communication stream as soon as the stage's last kernel is done, overlapping the remaining
// backward.  AdamW waits for the last bucket and applies the 1/world scaling.
#include <dlfcn.h>

#include <sched.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <vector>

#include "gen_model.h"

namespace wb {

namespace {

// Minimal NCCL ABI (stable since NCCL 2.x).
typedef struct ncclComm* ncclComm_t;
typedef struct {
  char internal[128];
} ncclUniqueId;
typedef enum { ncclSuccess = 0, ncclInProgress = 7 } ncclResult_t;
enum { ncclFloat32 = 7 };
enum { ncclSum = 0 };

struct NcclApi {
  void* h = nullptr;
  int (*GetUniqueId)(ncclUniqueId*) = nullptr;
  int (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  int (*AllReduce)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
  int (*CommDestroy)(ncclComm_t) = nullptr;
  int (*CommAbort)(ncclComm_t) = nullptr;
  int (*CommGetAsyncError)(ncclComm_t, int*) = nullptr;
  const char* (*GetErrorString)(int) = nullptr;
  bool ok = false;
};

NcclApi& nccl() {
  static NcclApi api;
  static bool tried = false;
  if (tried) return api;
  tried = true;
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char* n : names) {
    api.h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (api.h) break;
  }
  if (!api.h) {
    fprintf(stderr, "wuburvc_b200: libnccl.so.2 not found (%s)\n", dlerror());
    return api;
  }
  api.GetUniqueId = (int (*)(ncclUniqueId*))dlsym(api.h, "ncclGetUniqueId");
  api.CommInitRank = (int (*)(ncclComm_t*, int, ncclUniqueId, int))dlsym(api.h, "ncclCommInitRank");
  api.AllReduce = (int (*)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t))dlsym(api.h, "ncclAllReduce");
  api.CommDestroy = (int (*)(ncclComm_t))dlsym(api.h, "ncclCommDestroy");
  api.CommAbort = (int (*)(ncclComm_t))dlsym(api.h, "ncclCommAbort");
  api.CommGetAsyncError = (int (*)(ncclComm_t, int*))dlsym(api.h, "ncclCommGetAsyncError");
  api.GetErrorString = (const char* (*)(int))dlsym(api.h, "ncclGetErrorString");
  api.ok = api.GetUniqueId && api.CommInitRank && api.AllReduce && api.CommDestroy;
  return api;
}

}  // namespace

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  cudaStream_t cs = nullptr;
  cudaEvent_t done = nullptr;
  std::vector<cudaEvent_t> ready;           // one per bucket, recorded on the main stream
  std::vector<std::pair<long long, long long>> buckets;  // [off, end) in floats
  int timeout_ms = 60000;  // a step's collectives must finish within this (comm_sync)
  bool aborted = false;    // the communicator was aborted: the context runs no further step
};

// Bucket boundaries: end of conv_post + stage 3, stage 2, stage 1, stage 0, and the rest.
// Gradient all-reduce buckets, in the order the backward finishes them: stage 3's parameters, then
// stages 2, 1, 0 (each ends at its ups layer), then everything else (conv_pre, cond, source).  The
// flat buffer is laid out in that order, so bucket b is the contiguous range [first, second).  Every
// bucket is kept (possibly empty) so that bucket index b always means stage 3 - b.
static std::vector<std::pair<long long, long long>> plan_buckets(const ParamTable& t) {
  std::vector<long long> ends;
  for (int L = 3; L >= 0; --L) {
    const std::string key = "dec.ups." + std::to_string(L) + ".bias";
    long long end = 0;
    for (const auto& e : t.e)
      if (e.name == key || e.name == "dec.ups_act." + std::to_string(L) + ".alpha") end = std::max(end, e.off + e.n);
    ends.push_back((end + 63) / 64 * 64);
  }
  ends.push_back(t.total);
  std::vector<std::pair<long long, long long>> b;
  long long prev = 0;
  for (long long e : ends) {
    const long long end = std::min(std::max(e, prev), t.total);
    b.push_back({prev, end});
    prev = end;
  }
  return b;
}

// The context's buckets: the last one also carries the range-flag slot after the gradients (4 floats,
// keeping the bucket a multiple of 16 bytes), so every rank learns whether any rank's forward overflowed.
static std::vector<std::pair<long long, long long>> make_buckets(const Gen& m) {
  auto b = plan_buckets(m.table);
  b.back().second = m.table.total + 4;
  return b;
}

}  // namespace wb

int wubu_b200_gen_bucket_plan(const WubuB200GenConfig* cfg, long long* ends, int cap) {
  using namespace wb;
  if (!cfg || !config_valid(*cfg)) return WUBU_B200_ERR_ARG;
  const ParamTable t = build_param_table(*cfg);
  if (t.e.empty()) return WUBU_B200_ERR_ARG;
  const auto b = plan_buckets(t);
  if (ends) {
    if (cap < (int)b.size()) return WUBU_B200_ERR_ARG;
    for (size_t i = 0; i < b.size(); ++i) ends[i] = b[i].second;
  }
  return (int)b.size();
}

namespace wb {

int comm_bucket_count(Gen& m) { return m.comm ? (int)m.comm->buckets.size() : 0; }

// Called once bucket `b`'s gradients are final on stream `producer`: the comm stream waits for
// them and all-reduces them in place.
int comm_bucket_ready(Gen& m, int b, cudaStream_t producer) {
  Comm* c = m.comm;
  if (!c || c->world <= 1) return 0;
  if (c->aborted) return WUBU_B200_ERR_COMM;
  NcclApi& api = nccl();
  if (b + 1 == (int)c->buckets.size()) range_flag(m.err, m.grads + m.table.total, producer);
  if (cudaEventRecord(c->ready[b], producer) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  if (cudaStreamWaitEvent(c->cs, c->ready[b], 0) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  const auto& r = c->buckets[b];
  if (r.second <= r.first) return 0;  // empty bucket: every rank skips it alike
  const int rc = api.AllReduce(m.grads + r.first, m.grads + r.first, (size_t)(r.second - r.first), ncclFloat32,
                               ncclSum, c->comm, c->cs);
  if (rc != ncclSuccess) {
    fprintf(stderr, "wuburvc_b200: ncclAllReduce failed: %s\n", api.GetErrorString ? api.GetErrorString(rc) : "?");
    return WUBU_B200_ERR_COMM;
  }
  return 0;
}

// Main stream waits for every bucket (before AdamW).
int comm_join(Gen& m) {
  Comm* c = m.comm;
  if (!c || c->world <= 1) return 0;
  if (cudaEventRecord(c->done, c->cs) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  if (cudaStreamWaitEvent(m.stream, c->done, 0) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  return 0;
}

int comm_world(Gen& m) { return m.comm ? m.comm->world : 1; }

bool comm_aborted(Gen& m) { return m.comm && m.comm->aborted; }

int comm_set_timeout(Gen& m, int ms) {
  if (!m.comm || ms <= 0) return WUBU_B200_ERR_ARG;
  m.comm->timeout_ms = ms;
  return 0;
}

// Waits for the model stream of a context with a communicator.  The stream and the communicator's
// asynchronous error are polled; past the deadline (a peer that hangs or left mid-step) or on an
// NCCL error, the communicator is aborted, which ends the collectives waiting on the peer, and the
// call reports WUBU_B200_ERR_COMM.  The context then runs no further step (its captured step holds
// the aborted communicator).
int comm_sync(Gen& m) {
  Comm* c = m.comm;
  NcclApi& api = nccl();
  const auto t0 = std::chrono::steady_clock::now();
  auto fail = [&](const char* why) {
    fprintf(stderr, "wuburvc_b200: %s: aborting the communicator\n", why);
    if (api.CommAbort && c->comm) api.CommAbort(c->comm);
    c->comm = nullptr;
    c->aborted = true;
    cudaStreamSynchronize(m.stream);  // the aborted collectives have ended
    cudaGetLastError();
    return WUBU_B200_ERR_COMM;
  };
  for (long long spins = 0;; ++spins) {
    const cudaError_t q = cudaStreamQuery(m.stream);
    if (q == cudaSuccess) return 0;
    if (q != cudaErrorNotReady) return WUBU_B200_ERR_CUDA;
    if (api.CommGetAsyncError && c->comm) {
      int ae = ncclSuccess;
      if (api.CommGetAsyncError(c->comm, &ae) == ncclSuccess && ae != ncclSuccess && ae != ncclInProgress)
        return fail(api.GetErrorString ? api.GetErrorString(ae) : "NCCL asynchronous error");
    }
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (ms.count() > c->timeout_ms) return fail("the step's collectives did not finish within the comm timeout");
    if (spins < 20000) sched_yield();
    else usleep(50);
  }
}

int comm_allreduce_grads(Gen& m) {
  for (int b = 0; b < comm_bucket_count(m); ++b) {
    const int rc = comm_bucket_ready(m, b, m.stream);
    if (rc) return rc;
  }
  return comm_join(m);
}

void comm_destroy(Gen& m) {
  if (!m.comm) return;
  Comm* c = m.comm;
  NcclApi& api = nccl();
  if (c->cs) cudaStreamSynchronize(c->cs);
  if (c->comm && api.CommDestroy) api.CommDestroy(c->comm);
  for (auto e : c->ready) cudaEventDestroy(e);
  if (c->done) cudaEventDestroy(c->done);
  if (c->cs) cudaStreamDestroy(c->cs);
  delete m.comm;
  m.comm = nullptr;
}

int comm_attach(Gen& m, int rank, int world, const void* id128) {
  if (world < 1 || rank < 0 || rank >= world || !id128) return WUBU_B200_ERR_ARG;
  comm_destroy(m);
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world;
  c->buckets = make_buckets(m);
  if (world > 1) {
    NcclApi& api = nccl();
    if (!api.ok) return WUBU_B200_ERR_COMM;
    ncclUniqueId id;
    memcpy(&id, id128, sizeof(id));
    cudaSetDevice(m.opt.device);
    const int rc = api.CommInitRank(&c->comm, world, id, rank);
    if (rc != ncclSuccess) {
      fprintf(stderr, "wuburvc_b200: ncclCommInitRank failed: %s\n", api.GetErrorString ? api.GetErrorString(rc) : "?");
      return WUBU_B200_ERR_COMM;
    }
  }
  if (cudaStreamCreateWithFlags(&c->cs, cudaStreamNonBlocking) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  c->ready.resize(c->buckets.size());
  for (auto& e : c->ready)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  if (cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  m.comm = c;
  return 0;
}

int comm_unique_id(void* out128) {
  NcclApi& api = nccl();
  if (!api.ok) return WUBU_B200_ERR_COMM;
  ncclUniqueId id;
  if (api.GetUniqueId(&id) != ncclSuccess) return WUBU_B200_ERR_COMM;
  memcpy(out128, &id, sizeof(id));
  return 0;
}

// A plain communicator on the same NCCL (the discriminators' gradient all-reduce).
int nccl_plain_init(void** out, int rank, int world, const void* id128) {
  NcclApi& api = nccl();
  if (!out || !id128 || world < 2 || rank < 0 || rank >= world) return WUBU_B200_ERR_ARG;
  if (!api.ok) return WUBU_B200_ERR_COMM;
  ncclUniqueId id;
  memcpy(&id, id128, sizeof(id));
  ncclComm_t c = nullptr;
  const int rc = api.CommInitRank(&c, world, id, rank);
  if (rc != ncclSuccess) {
    fprintf(stderr, "wuburvc_b200: ncclCommInitRank failed: %s\n", api.GetErrorString ? api.GetErrorString(rc) : "?");
    return WUBU_B200_ERR_COMM;
  }
  *out = c;
  return 0;
}

int nccl_plain_allreduce_sum(void* comm, float* buf, size_t n, cudaStream_t st) {
  NcclApi& api = nccl();
  const int rc = api.AllReduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st);
  if (rc != ncclSuccess) {
    fprintf(stderr, "wuburvc_b200: ncclAllReduce failed: %s\n", api.GetErrorString ? api.GetErrorString(rc) : "?");
    return WUBU_B200_ERR_COMM;
  }
  return 0;
}

// 0, or WUBU_B200_ERR_COMM when the communicator reports an asynchronous error
int nccl_plain_async_error(void* comm) {
  NcclApi& api = nccl();
  int ae = ncclSuccess;
  if (api.CommGetAsyncError && api.CommGetAsyncError(static_cast<ncclComm_t>(comm), &ae) == ncclSuccess &&
      ae != ncclSuccess && ae != ncclInProgress)
    return WUBU_B200_ERR_COMM;
  return 0;
}

void nccl_plain_abort(void* comm) {
  NcclApi& api = nccl();
  if (comm && api.CommAbort) api.CommAbort(static_cast<ncclComm_t>(comm));
}

void nccl_plain_destroy(void* comm) {
  NcclApi& api = nccl();
  if (comm && api.CommDestroy) api.CommDestroy(static_cast<ncclComm_t>(comm));
}

}  // namespace wb
