// peer_exchange.cu -- the tensor-parallel sampler's exchange rounds over
// NVLink peer memory instead of NCCL collectives.
//
// DistributedContext (src/distributed.rs:61-98) shards the vocabulary; the
// sharded acceptance then needs three small exchanges per step (row maxima
// with the normaliser parts under them, weight totals, the sampled token),
// each a few KB to a few hundred KB.  At that size an NCCL collective costs
// its launch and protocol latency (~20 us a round measured on two B200s).  Here every rank
// maps every peer's exchange region once (CUDA IPC, at kyro_ctx_tp_init) and
// one kernel per round stores this rank's payload straight into each peer's
// region over NVLink, raises a per-sender flag there, and waits for the
// peers' flags on its own.
//
// The region's layout is in xchg.cuh.  Round 1 of the sampler is stored by
// its producer kernel straight into the peers' slots (sampler.cu); the
// other rounds run through the exchange kernel below.
//
// Rounds are numbered on the device (the counter), so a captured CUDA graph
// replays with fresh numbers.  A slot of parity s is written again only in
// round s + 2, which a sender starts after it has seen the receiver's flag
// of round s + 1, raised after the receiver's round-s kernel had finished
// reading the slot.  Flags are kept per parity for the same reason: a peer
// can be one round ahead (it finishes round s as soon as this rank's flag
// lands, then raises its round-(s+1) flag), but never two, so a wait on the
// parity-s flag sees round s or nothing, and a peer that skipped round s
// cannot satisfy it with its next round's flag.
//
// Every wait is bounded: a flag that does not arrive within the context's
// wait bound (kyro_ctx_set_wait_timeout; 2 s unless KYRO_WAIT_TIMEOUT_MS
// says otherwise) sets KYRO_DEV_WAIT_TIMEOUT in the status word and the
// kernel returns.  After a timeout the ranks' round counters no longer
// agree and a late peer may still write into a slot that will be reused,
// so the context must be destroyed and the group formed again.
#include <cstdlib>
#include <cstring>

#include "kyro_internal.cuh"
#include "xchg.cuh"

namespace {

using kyro::xchg::flag_of;
using kyro::xchg::globaltimer;
using kyro::xchg::kCtlBytes;
using kyro::xchg::kHalfBytes;
using kyro::xchg::kSeqOffset;
using kyro::xchg::ld_acquire_sys;
using kyro::xchg::Peers;
using kyro::xchg::st_release_sys;

constexpr int kXchgThreads = 512;

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Copy `bytes` (a multiple of 4) from src to dst with the block's threads,
// 16 bytes at a time when both ends and the size allow it.
__device__ __forceinline__ void copy_words(uint8_t* dst, const uint8_t* src, size_t bytes) {
  if (((uintptr_t)dst | (uintptr_t)src | bytes) % 16 == 0) {
    const size_t n = bytes / 16;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    const size_t n = bytes / 4;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x)
      reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
  }
}

// One cluster of `world` CTAs; CTA p talks to rank p.  mode 0: recv gets the
// world * bytes concatenation of every rank's payload (slot order = rank
// order).  mode 1: recv[i] = max over ranks of the int32 payload element i.
// A wait for a peer's flag gives up after wait_ns nanoseconds.  skip is
// fault injection for the tests (always 0 otherwise): 1 makes this rank
// skip the round towards its peers while staying alive (it neither stores
// its payload in their regions nor raises their flags, so a peer waiting
// for them runs into its bound); 2 skips its own slot as well, so that a
// one-rank group waits for a flag that nothing sets.
__global__ void __launch_bounds__(kXchgThreads)
peer_exchange_kernel(Peers peers, int rank, int world, const uint8_t* __restrict__ send,
                     uint8_t* __restrict__ recv, size_t bytes, int mode, uint32_t* status,
                     unsigned long long wait_ns, int skip) {
  const int p = blockIdx.x;  // == the CTA's rank in the cluster (the grid is one cluster)
  uint8_t* own = peers.p[rank];
  unsigned long long* ctr = reinterpret_cast<unsigned long long*>(own + kSeqOffset);
  kyro::dev::pdl_wait();
  // the consumer of recv may begin launching now: it waits for this grid to
  // complete before it reads
  kyro::dev::pdl_trigger();
  // every CTA reads the round number before CTA 0 advances it
  const unsigned long long seq = *reinterpret_cast<volatile unsigned long long*>(ctr) + 1ull;
  cluster_sync_all();
  if (p == 0 && threadIdx.x == 0) *ctr = seq;
  const size_t half = (seq & 1ull) * kHalfBytes;
  // this rank's payload into rank p's slot `rank`
  const size_t stride = (bytes + 15) & ~size_t(15);  // slots start 16-byte aligned
  const bool send_p = skip == 0 || (skip == 1 && p == rank);
  if (send_p) copy_words(peers.p[p] + kCtlBytes + half + (size_t)rank * stride, send, bytes);
  __threadfence_system();
  __syncthreads();
  __shared__ int timed_out;
  if (threadIdx.x == 0) {
    timed_out = 0;
    if (send_p) st_release_sys(flag_of(peers.p[p], rank, seq), seq);
    // rank p's payload for this round has landed here once its flag of this
    // round's parity reads seq
    const unsigned long long* flag = flag_of(own, p, seq);
    const unsigned long long t0 = globaltimer();
    while (ld_acquire_sys(flag) < seq) {
      if (globaltimer() - t0 > wait_ns) {
        kyro::dev::flag(status, KYRO_DEV_WAIT_TIMEOUT);
        timed_out = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  const uint8_t* slots = own + kCtlBytes + half;
  if (mode == 0) {
    if (!timed_out) copy_words(recv + (size_t)p * bytes, slots + (size_t)p * stride, bytes);
  }
  // every CTA has waited for its sender (and copied its slot) past here
  cluster_sync_all();
  if (mode == 1 && p == 0) {
    const size_t n = bytes / 4;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
      int32_t m = reinterpret_cast<const int32_t*>(slots)[i];
      for (int r = 1; r < world; ++r)
        m = max(m, reinterpret_cast<const int32_t*>(slots + (size_t)r * stride)[i]);
      reinterpret_cast<int32_t*>(recv)[i] = m;
    }
  }
}

bool forced_nccl() {
  const char* e = getenv("KYRO_TP_TRANSPORT");
  return e && strcmp(e, "nccl") == 0;
}

}  // namespace

namespace kyro {
namespace xchg {

// What each rank contributes to the setup: its region's IPC handle, whether
// it has one, and its GPU's UUID (ranks that share a GPU keep NCCL: their
// exchange kernels would wait on one another on one device).
struct SetupRec {
  cudaIpcMemHandle_t handle;
  unsigned char uuid[16];
  int32_t ok;
  int32_t pad[11];
};

size_t setup_bytes(int world) { return sizeof(SetupRec) * (size_t)(world + 1) + 64; }

int init(kyro_ctx* ctx, uint8_t* dh) {
  ctx->xchg_ready = false;
  ctx->xchg_local = nullptr;
  for (int r = 0; r < KYRO_MAX_TP_WORLD; ++r) ctx->xchg_peer[r] = nullptr;
  const int world = ctx->tp_world;
  if (world <= 1 || world > KYRO_MAX_TP_WORLD) return KYRO_OK;
  // Every rank takes the same two collectives below whatever happens locally,
  // so that a rank that cannot use the peer path never leaves the others
  // waiting; the group then agrees to keep NCCL.
  SetupRec mine;
  memset(&mine, 0, sizeof(mine));
  mine.ok = forced_nccl() ? 0 : 1;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, ctx->device) == cudaSuccess)
    memcpy(mine.uuid, &prop.uuid, sizeof(mine.uuid));
  else
    mine.ok = 0;
  const size_t region = kCtlBytes + 2 * kHalfBytes;
  uint8_t* local = nullptr;
  if (mine.ok && cudaMalloc(&local, region) != cudaSuccess) {
    local = nullptr;
    mine.ok = 0;
  }
  if (mine.ok && (cudaMemset(local, 0, region) != cudaSuccess ||
                  cudaIpcGetMemHandle(&mine.handle, local) != cudaSuccess))
    mine.ok = 0;
  cudaGetLastError();
  // The setup's collectives run synchronously on a private stream, or on the
  // context's own stream if no stream can be made.  `dh` (the exchange
  // records) was allocated by the caller before the group formed, so no
  // local failure from here on skips a collective.
  cudaStream_t saved = ctx->stream, s = nullptr;
  const bool own_stream = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess;
  if (!own_stream) {
    cudaGetLastError();
    s = saved;
  }
  ctx->stream = s;
  cudaError_t err;
  uint8_t* d_mine = dh + sizeof(SetupRec) * world;
  cudaMemcpy(d_mine, &mine, sizeof(mine), cudaMemcpyHostToDevice);
  int st = nccl::all_gather(ctx, d_mine, dh, sizeof(SetupRec), "peer exchange setup");
  if (st == KYRO_OK) {
    err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) st = cuda_error(err, "cudaStreamSynchronize(peer exchange setup)");
  }
  SetupRec all[KYRO_MAX_TP_WORLD];
  if (st == KYRO_OK) cudaMemcpy(all, dh, sizeof(SetupRec) * world, cudaMemcpyDeviceToHost);
  bool ok = st == KYRO_OK;
  for (int r = 0; ok && r < world; ++r) {
    ok = all[r].ok != 0;
    for (int q = 0; ok && q < r; ++q) ok = memcmp(all[q].uuid, all[r].uuid, 16) != 0;
  }
  for (int r = 0; ok && r < world; ++r) {
    if (r == ctx->tp_rank) {
      ctx->xchg_peer[r] = local;
      continue;
    }
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[r].handle, cudaIpcMemLazyEnablePeerAccess) !=
        cudaSuccess) {
      cudaGetLastError();
      ok = false;
      break;
    }
    ctx->xchg_peer[r] = (uint8_t*)ptr;
  }
  // agreement: every rank mapped every peer
  int32_t agreed = 0;
  if (st == KYRO_OK) {
    const int32_t flag = ok ? 1 : 0;
    cudaMemcpy(dh, &flag, 4, cudaMemcpyHostToDevice);
    st = nccl::all_reduce_min_i32(ctx, (const int32_t*)dh, (int32_t*)(dh + 16), 1,
                                  "peer exchange agreement");
    if (st == KYRO_OK) {
      err = cudaStreamSynchronize(s);
      if (err != cudaSuccess) st = cuda_error(err, "cudaStreamSynchronize(peer exchange agreement)");
    }
    if (st == KYRO_OK) cudaMemcpy(&agreed, dh + 16, 4, cudaMemcpyDeviceToHost);
  }
  ctx->stream = saved;
  if (own_stream) cudaStreamDestroy(s);
  if (st != KYRO_OK || !agreed) {
    for (int r = 0; r < world; ++r)
      if (r != ctx->tp_rank && ctx->xchg_peer[r]) cudaIpcCloseMemHandle(ctx->xchg_peer[r]);
    for (int r = 0; r < KYRO_MAX_TP_WORLD; ++r) ctx->xchg_peer[r] = nullptr;
    if (local) cudaFree(local);
    return st;
  }
  ctx->xchg_local = local;
  ctx->xchg_ready = true;
  return KYRO_OK;
}

void release(kyro_ctx* ctx) {
  if (!ctx->xchg_ready) return;
  for (int r = 0; r < ctx->tp_world; ++r)
    if (r != ctx->tp_rank && ctx->xchg_peer[r]) cudaIpcCloseMemHandle(ctx->xchg_peer[r]);
  cudaFree(ctx->xchg_local);
  ctx->xchg_local = nullptr;
  for (int r = 0; r < KYRO_MAX_TP_WORLD; ++r) ctx->xchg_peer[r] = nullptr;
  ctx->xchg_ready = false;
}

static int launch(kyro_ctx* ctx, const void* send, void* recv, size_t bytes, int mode,
                  const char* what) {
  int skip = 0;
  if (ctx->xchg_skip_rounds > 0) {  // fault injection: this rank skips the round
    --ctx->xchg_skip_rounds;
    skip = 1;
  }
  Peers peers = {};
  for (int r = 0; r < ctx->tp_world; ++r) peers.p[r] = ctx->xchg_peer[r];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctx->tp_world);
  cfg.blockDim = dim3(kXchgThreads);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)ctx->tp_world;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err =
      cudaLaunchKernelEx(&cfg, peer_exchange_kernel, peers, ctx->tp_rank, ctx->tp_world,
                         (const uint8_t*)send, (uint8_t*)recv, bytes, mode, ctx->d_status,
                         (unsigned long long)ctx->wait_ns, skip);
  if (err != cudaSuccess) return cuda_error(err, what);
  return KYRO_OK;
}

bool fits(kyro_ctx* ctx, size_t bytes) {
  return ctx->xchg_ready && bytes % 4 == 0 &&
         ((bytes + 15) & ~size_t(15)) * (size_t)ctx->tp_world <= kHalfBytes;
}

bool push_round(kyro_ctx* ctx, size_t bytes, Peers* peers, int* skip) {
  if (!fits(ctx, bytes)) return false;
  *skip = 0;
  if (ctx->xchg_skip_rounds > 0) {  // fault injection: this rank skips the round
    --ctx->xchg_skip_rounds;
    *skip = 1;
  }
  for (int r = 0; r < KYRO_MAX_TP_WORLD; ++r)
    peers->p[r] = r < ctx->tp_world ? ctx->xchg_peer[r] : nullptr;
  return true;
}

int all_gather(kyro_ctx* ctx, const void* send, void* recv, size_t bytes, const char* what) {
  if (!fits(ctx, bytes))
    return nccl::all_gather(ctx, send, recv, bytes, what);
  KY_REQUIRE((uintptr_t)send % 4 == 0 && (uintptr_t)recv % 4 == 0,
             "%s: exchange buffers must be 4-byte aligned", what);
  return launch(ctx, send, recv, bytes, 0, what);
}

int all_reduce_max_i32(kyro_ctx* ctx, const int32_t* send, int32_t* recv, size_t count,
                       const char* what) {
  const size_t bytes = count * 4;
  if (!fits(ctx, bytes))
    return nccl::all_reduce_max_i32(ctx, send, recv, count, what);
  KY_REQUIRE((uintptr_t)send % 4 == 0 && (uintptr_t)recv % 4 == 0,
             "%s: exchange buffers must be 4-byte aligned", what);
  return launch(ctx, send, recv, bytes, 1, what);
}

}  // namespace xchg
}  // namespace kyro

// ---------------------------------------------------------------- self-test
//
// The exchange kernel's bounded wait, run on one GPU: a one-rank "group"
// over a caller-given region, with the round skipped, so the kernel waits
// for a flag that nothing sets.  It must give up after the context's wait
// bound, set KYRO_DEV_WAIT_TIMEOUT and return; the context stays usable.
extern "C" int kyro_selftest_exchange_timeout(kyro_ctx* ctx, void* region, size_t region_bytes) {
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(region && region_bytes >= kCtlBytes && (uintptr_t)region % 256 == 0,
             "kyro_selftest_exchange_timeout: region must be 256-byte aligned and hold %zu bytes",
             kCtlBytes);
  cudaError_t err = cudaMemsetAsync(region, 0, kCtlBytes, ctx->stream);
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaMemsetAsync(self-test region)");
  Peers peers = {};
  peers.p[0] = (uint8_t*)region;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kXchgThreads);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, peer_exchange_kernel, peers, 0, 1, (const uint8_t*)nullptr,
                           (uint8_t*)nullptr, (size_t)0, 0, ctx->d_status,
                           (unsigned long long)ctx->wait_ns, 2);
  if (err != cudaSuccess) return kyro::cuda_error(err, "peer_exchange_kernel (self-test)");
  return KYRO_OK;
}

extern "C" int kyro_ctx_tp_inject_skip(kyro_ctx* ctx, int32_t rounds) {
  if (!ctx) return kyro::set_error(KYRO_ERR_INVALID_ARG, "null kyro_ctx");
  KY_REQUIRE(rounds >= 0, "kyro_ctx_tp_inject_skip: rounds = %d", rounds);
  KY_REQUIRE(ctx->xchg_ready, "kyro_ctx_tp_inject_skip: the context's exchange is not on peer memory");
  ctx->xchg_skip_rounds = rounds;
  return KYRO_OK;
}
