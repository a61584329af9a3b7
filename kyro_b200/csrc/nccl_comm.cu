// nccl_comm.cu -- the tensor-parallel group of a context.
//
// The reference's DistributedContext::all_reduce (src/distributed.rs:61-79)
// is a stub that returns its input.  Here the vocabulary-sharded acceptance
// step exchanges a few bytes per row over NCCL.  NCCL is opened at run time
// (dlopen), so the library loads, and everything but the TP entry points
// works, on a machine without it; the TP entry points fail with
// KYRO_ERR_NCCL and a message naming the library they looked for.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "kyro_internal.cuh"
#include "watchdog.h"

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

std::once_flag g_once;
NcclApi g_api;
bool g_ok = false;
char g_why[512];

void load_api() {
  const char* path = std::getenv("KYRO_NCCL_LIBRARY");
  if (!path || !*path) path = "libnccl.so.2";
  void* h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    snprintf(g_why, sizeof(g_why), "cannot open %s: %s", path, dlerror());
    return;
  }
  bool ok = true;
  auto sym = [&](const char* name) {
    void* f = dlsym(h, name);
    if (!f) ok = false;
    return f;
  };
  g_api.GetUniqueId = (decltype(g_api.GetUniqueId))sym("ncclGetUniqueId");
  g_api.CommInitRank = (decltype(g_api.CommInitRank))sym("ncclCommInitRank");
  g_api.CommDestroy = (decltype(g_api.CommDestroy))sym("ncclCommDestroy");
  g_api.CommAbort = (decltype(g_api.CommAbort))sym("ncclCommAbort");
  g_api.AllGather = (decltype(g_api.AllGather))sym("ncclAllGather");
  g_api.AllReduce = (decltype(g_api.AllReduce))sym("ncclAllReduce");
  g_api.GetErrorString = (decltype(g_api.GetErrorString))sym("ncclGetErrorString");
  if (!ok) {
    snprintf(g_why, sizeof(g_why), "%s lacks an NCCL entry point", path);
    return;
  }
  g_ok = true;
}

const NcclApi* api() {
  std::call_once(g_once, load_api);
  return g_ok ? &g_api : nullptr;
}

int nccl_error(ncclResult_t r, const char* what) {
  const NcclApi* a = api();
  return kyro::set_error(KYRO_ERR_NCCL, "%s: %s", what,
                         a ? a->GetErrorString(r) : "NCCL error");
}

int need_api(const NcclApi** out, const char* what) {
  *out = api();
  if (!*out) return kyro::set_error(KYRO_ERR_NCCL, "%s: NCCL unavailable (%s)", what, g_why);
  return KYRO_OK;
}

// The context's host watchdog over its NCCL collectives: a ring of CUDA
// events, one recorded after each sharded call's collectives; a call whose
// event has not completed within the context's wait bound gets the
// communicator aborted (ncclCommAbort ends the stuck collectives), and the
// context's TP calls fail from then on.
constexpr int kWatchEvents = 64;

struct NcclWatch {
  kyro_ctx* ctx;
  cudaEvent_t ev[kWatchEvents];
  int next;
  kyro::Watchdog* wd;
};

int watch_poll(void* user, void* probe) {
  (void)user;
  return cudaEventQuery((cudaEvent_t)probe) != cudaErrorNotReady;
}

void watch_abort(void* user) {
  NcclWatch* w = (NcclWatch*)user;
  const NcclApi* a = api();
  if (a && w->ctx->nccl_comm) a->CommAbort((ncclComm_t)w->ctx->nccl_comm);
  w->ctx->tp_aborted = 1;
}

void watch_setup(void* user) { cudaSetDevice(((NcclWatch*)user)->ctx->device); }

int start_watch(kyro_ctx* ctx) {
  NcclWatch* w = new NcclWatch();
  w->ctx = ctx;
  w->next = 0;
  for (int i = 0; i < kWatchEvents; ++i) {
    const cudaError_t err = cudaEventCreateWithFlags(&w->ev[i], cudaEventDisableTiming);
    if (err != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(w->ev[j]);
      delete w;
      return kyro::cuda_error(err, "cudaEventCreate(NCCL watchdog)");
    }
  }
  w->wd = new kyro::Watchdog(watch_poll, watch_abort, watch_setup, w);
  ctx->watchdog = w;
  return KYRO_OK;
}

void stop_watch(kyro_ctx* ctx) {
  NcclWatch* w = (NcclWatch*)ctx->watchdog;
  if (!w) return;
  delete w->wd;  // joins the thread
  for (int i = 0; i < kWatchEvents; ++i) cudaEventDestroy(w->ev[i]);
  delete w;
  ctx->watchdog = nullptr;
}

}  // namespace

namespace kyro {
namespace nccl {

void watch(kyro_ctx* ctx) {
  NcclWatch* w = (NcclWatch*)ctx->watchdog;
  if (!w) return;
  // a captured graph's replays run outside these calls: not watched
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(ctx->stream, &cs) != cudaSuccess ||
      cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return;
  }
  cudaEvent_t ev = w->ev[w->next % kWatchEvents];
  if (w->wd->pending((void*)ev)) return;  // 64 calls still in flight: this one goes unwatched
  ++w->next;
  if (cudaEventRecord(ev, ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  w->wd->arm((void*)ev, ctx->wait_ns);
}

int all_gather(kyro_ctx* ctx, const void* send, void* recv, size_t bytes, const char* what) {
  const NcclApi* a;
  KY_TRY(need_api(&a, what));
  const ncclResult_t r =
      a->AllGather(send, recv, bytes, ncclUint8, (ncclComm_t)ctx->nccl_comm, ctx->stream);
  return r == ncclSuccess ? KYRO_OK : nccl_error(r, what);
}

int all_reduce_max_i32(kyro_ctx* ctx, const int32_t* send, int32_t* recv, size_t count,
                       const char* what) {
  const NcclApi* a;
  KY_TRY(need_api(&a, what));
  const ncclResult_t r = a->AllReduce(send, recv, count, ncclInt32, ncclMax,
                                      (ncclComm_t)ctx->nccl_comm, ctx->stream);
  return r == ncclSuccess ? KYRO_OK : nccl_error(r, what);
}

int all_reduce_min_i32(kyro_ctx* ctx, const int32_t* send, int32_t* recv, size_t count,
                       const char* what) {
  const NcclApi* a;
  KY_TRY(need_api(&a, what));
  const ncclResult_t r = a->AllReduce(send, recv, count, ncclInt32, ncclMin,
                                      (ncclComm_t)ctx->nccl_comm, ctx->stream);
  return r == ncclSuccess ? KYRO_OK : nccl_error(r, what);
}

void release(kyro_ctx* ctx) {
  stop_watch(ctx);
  xchg::release(ctx);
  if (!ctx->nccl_comm) return;
  const NcclApi* a = api();
  // an aborted communicator is already gone
  if (a && !ctx->tp_aborted) a->CommDestroy((ncclComm_t)ctx->nccl_comm);
  ctx->nccl_comm = nullptr;
  ctx->tp_rank = 0;
  ctx->tp_world = 1;
}

}  // namespace nccl
}  // namespace kyro

extern "C" int kyro_tp_unique_id(void* out) {
  if (!out) return kyro::set_error(KYRO_ERR_INVALID_ARG, "kyro_tp_unique_id: out is NULL");
  const NcclApi* a;
  KY_TRY(need_api(&a, "kyro_tp_unique_id"));
  static_assert(sizeof(ncclUniqueId) == KYRO_TP_UNIQUE_ID_BYTES, "NCCL unique id size");
  ncclUniqueId id;
  const ncclResult_t r = a->GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_error(r, "ncclGetUniqueId");
  memcpy(out, &id, sizeof(id));
  return KYRO_OK;
}

extern "C" int kyro_ctx_tp_init(kyro_ctx* ctx, const void* unique_id, int rank, int world) {
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(unique_id, "kyro_ctx_tp_init: unique_id is NULL");
  KY_REQUIRE(world >= 1 && rank >= 0 && rank < world, "kyro_ctx_tp_init: rank %d of %d", rank,
             world);
  KY_REQUIRE(!ctx->nccl_comm, "kyro_ctx_tp_init: the context already has a group");
  const NcclApi* a;
  KY_TRY(need_api(&a, "kyro_ctx_tp_init"));
  // The peer-exchange setup's device buffer is allocated before the group
  // forms: a failure here returns before the first collective, like an
  // argument error, and nothing after it can skip one of the setup's
  // collectives that the other ranks take.
  uint8_t* dh = nullptr;
  const cudaError_t err = cudaMalloc(&dh, kyro::xchg::setup_bytes(world));
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaMalloc(peer exchange setup)");
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  const ncclResult_t r = a->CommInitRank(&comm, world, id, rank);
  if (r != ncclSuccess) {
    cudaFree(dh);
    return nccl_error(r, "ncclCommInitRank");
  }
  ctx->nccl_comm = comm;
  ctx->tp_rank = rank;
  ctx->tp_world = world;
  int st = kyro::xchg::init(ctx, dh);
  cudaFree(dh);
  // collectives that stay on NCCL get the host watchdog
  if (st == KYRO_OK && !ctx->xchg_ready) st = start_watch(ctx);
  return st;
}

// The watchdog alone, on the host, with the caller's probe and abort hook:
// arms one probe with a bound of timeout_ms and blocks until the probe
// reports completion (KYRO_OK) or the bound passes and the abort hook has
// run once (KYRO_ERR_TIMEOUT).  Needs no GPU.
namespace {
struct SelftestHooks {
  int (*poll)(void*);
  void (*on_abort)(void*);
  void* user;
};
int selftest_poll(void* u, void*) { return ((SelftestHooks*)u)->poll(((SelftestHooks*)u)->user); }
void selftest_abort(void* u) { ((SelftestHooks*)u)->on_abort(((SelftestHooks*)u)->user); }
}  // namespace

extern "C" int kyro_selftest_watchdog(uint32_t timeout_ms, int (*poll)(void* user),
                                      void (*on_abort)(void* user), void* user) {
  KY_REQUIRE(poll && on_abort, "kyro_selftest_watchdog: poll and on_abort are required");
  KY_REQUIRE(timeout_ms >= 1 && timeout_ms <= 600000, "kyro_selftest_watchdog: %u ms",
             timeout_ms);
  SelftestHooks hooks{poll, on_abort, user};
  bool fired;
  {
    kyro::Watchdog wd(selftest_poll, selftest_abort, nullptr, &hooks);
    wd.arm(&hooks, (uint64_t)timeout_ms * 1000000ull);
    fired = wd.wait_idle();
  }
  if (fired)
    return kyro::set_error(KYRO_ERR_TIMEOUT, "kyro_selftest_watchdog: the probe did not complete "
                                             "within %u ms; the abort hook ran", timeout_ms);
  return KYRO_OK;
}

extern "C" int kyro_ctx_tp_transport(kyro_ctx* ctx) {
  if (!ctx || !ctx->nccl_comm) return 0;
  return ctx->xchg_ready ? 2 : 1;
}
