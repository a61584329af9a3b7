// kyro_internal.cuh -- shared plumbing of the sm_100a verify-step library:
// the context object, host-side error reporting, device status word and
// small device helpers (warp reductions, bounded mbarrier waits).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/kyro_spec.h"

// NVTX (header-only v3): each entry point that enqueues work marks its host
// span with a named range, so a timeline tool shows the verify step's K1 /
// K2 / K3 calls beside their kernels.  Without a tool attached a range is
// one predicted branch.
#include <nvtx3/nvToolsExt.h>

#define KYRO_MAX_TP_WORLD 8
// counts of the acceptance pipeline kept in each context (sampler.cu)
#define KYRO_ZEROED_WS 8
#define KYRO_PIPE_COUNTS 128

struct kyro_ctx {
  int device;
  cudaStream_t stream;
  uint32_t* d_status;  // KYRO_DEV_* bits, atomically OR-ed by kernels
  int num_sms;
  // tensor-parallel group (kyro_ctx_tp_init); world 1 without one
  void* nccl_comm;     // ncclComm_t
  int tp_rank, tp_world;
  // verify attention's split tickets: a per-call epoch, and the last
  // workspace whose tickets this context has zeroed
  uint32_t attn_epoch;
  const void* attn_ws_zeroed;
  // workspaces whose stats unit counter this context has zeroed (the last
  // KYRO_ZEROED_WS seen)
  const void* stats_ws_zeroed[KYRO_ZEROED_WS];
  int stats_ws_next;
  // the acceptance pipeline's generation count and finished-sequence
  // count (device words owned by the context; sampler.cu), and the salt
  // of its record tags
  uint32_t* d_pipe_counts;
  uint32_t pipe_salt;
  // the sharded sampler's exchange rounds over NVLink peer memory
  // (peer_exchange.cu): this rank's region and every rank's mapping of it
  bool xchg_ready;
  uint8_t* xchg_local;
  uint8_t* xchg_peer[KYRO_MAX_TP_WORLD];
  int xchg_skip_rounds;  // fault injection: exchange rounds this rank skips
  // bound of every device-side wait on another rank, and of the host
  // watchdog on NCCL collectives (kyro_ctx_set_wait_timeout)
  uint64_t wait_ns;
  // host watchdog of the NCCL collectives (nccl_comm.cu); set once it has
  // aborted the communicator, after which TP calls fail
  void* watchdog;
  volatile int tp_aborted;
};

namespace kyro {

// Record `msg` as the calling thread's last error and return `status`.
int set_error(int status, const char* fmt, ...);
// Map a CUDA error to KYRO_ERR_CUDA with a message naming `what`.
int cuda_error(cudaError_t err, const char* what);
// Check for a launch error right after enqueueing kernels.
int check_launch(const char* what);
// Validate a context and make its device current.
int enter(kyro_ctx* ctx);
// The wait bound a new context starts with: KYRO_WAIT_TIMEOUT_MS, else 2 s.
uint64_t default_wait_ns();
// Drop the cached device address of kyro_spec_accept_static's scratch array
// on `device` (sampler.cu), so that the next call looks it up again.
void static_scratch_forget(int device);

// Tensor-core attention for many query rows per KV head (tree_attention.cu):
// whether a shape fills its 128-row tiles, and the launch.
bool tree_attention_eligible(const kyro_attn_params* p);
int tree_attention_launch(kyro_ctx* ctx, const kyro_attn_params* p, const void* q,
                          const void* k_cache, const void* v_cache, const int64_t* block_table,
                          const int64_t* context_lens, const uint64_t* tree_mask, void* out);

// The KV commit of an acceptance call's accepted slots, then the reserve of
// the next step's slots, as one launch on the context's stream
// (kv_commit.cu); check_commit_args validates the KV arguments first.
namespace kv {
int check_commit_args(const kyro_kv_params* p, int32_t num_new, int32_t num_new_next,
                      const int32_t* accept_len, const int64_t* block_table,
                      const int64_t* context_lens, const int32_t* free_stack,
                      const int32_t* free_top, const int32_t* ref_counts, const char* what);
int launch_commit_reserve(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                          int32_t num_new_next, const int32_t* accept_len, int64_t* block_table,
                          int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                          int32_t* ref_counts, int32_t* out_ok);
}  // namespace kv

// NCCL, loaded at run time (nccl_comm.cu).  Collectives enqueue on the
// context's stream over its tensor-parallel communicator.
namespace nccl {
// every rank receives the world * bytes concatenation of all ranks' `bytes`
int all_gather(kyro_ctx* ctx, const void* send, void* recv, size_t bytes, const char* what);
// element-wise max of int32 over the group
int all_reduce_max_i32(kyro_ctx* ctx, const int32_t* send, int32_t* recv, size_t count,
                       const char* what);
// element-wise min of int32 over the group
int all_reduce_min_i32(kyro_ctx* ctx, const int32_t* send, int32_t* recv, size_t count,
                       const char* what);
// destroy the context's communicator (no-op without one)
void release(kyro_ctx* ctx);
// put the collectives enqueued so far under the context's host watchdog
// (NCCL transport only; a no-op otherwise and during stream capture)
void watch(kyro_ctx* ctx);
}  // namespace nccl

// The sharded sampler's exchange rounds over NVLink peer memory
// (peer_exchange.cu), with NCCL as the transport when the ranks cannot map
// each other's memory or KYRO_TP_TRANSPORT=nccl.
namespace xchg {
// bytes of the device buffer init() exchanges its setup records through
size_t setup_bytes(int world);
// map every rank's exchange region (collective over the context's group);
// `dh` holds setup_bytes(world) bytes of device memory
int init(kyro_ctx* ctx, uint8_t* dh);
void release(kyro_ctx* ctx);
int all_gather(kyro_ctx* ctx, const void* send, void* recv, size_t bytes, const char* what);
// Whether the next round (a payload of `bytes` per rank) can be stored by its
// producer kernel straight into the peers' regions (xchg.cuh): fills
// `peers` and takes this rank's fault-injection skip for the round (1: it
// stores and flags only its own slot), as the exchange kernel would.
struct Peers;
bool push_round(kyro_ctx* ctx, size_t bytes, Peers* peers, int* skip);
int all_reduce_max_i32(kyro_ctx* ctx, const int32_t* send, int32_t* recv, size_t count,
                       const char* what);
}  // namespace xchg

}  // namespace kyro

namespace kyro {
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
}  // namespace kyro
#define KY_NVTX(name) kyro::NvtxRange ky_nvtx_range_(name)

#define KY_REQUIRE(cond, ...)                                       \
  do {                                                              \
    if (!(cond)) return kyro::set_error(KYRO_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define KY_TRY(expr)              \
  do {                            \
    int _st = (expr);             \
    if (_st != KYRO_OK) return _st; \
  } while (0)

// ---------------------------------------------------------------- device
namespace kyro {
// Launch `kernel` with programmatic stream serialization (see dev::pdl_wait).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               const char* name, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) return cuda_error(err, name);
  return KYRO_OK;
}

namespace dev {

__device__ __forceinline__ void flag(uint32_t* status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

// Programmatic dependent launch.  A kernel started with launch_pdl may run
// while its predecessor on the stream drains; pdl_wait blocks until that
// grid has completed and its writes are visible, so it comes before the
// kernel reads or writes anything a predecessor may touch.  pdl_trigger
// lets the next kernel begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// max value, lowest index among equal maxima
__device__ __forceinline__ void warp_argmax(float& v, int& idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
}

// Upper bound on the clock cycles any single device-side wait may take
// before the kernel records KYRO_DEV_WAIT_TIMEOUT and moves on (~1 s).
constexpr long long kWaitBudgetCycles = 2000000000ll;

}  // namespace dev
}  // namespace kyro
