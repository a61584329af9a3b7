// context.cu -- kyro_ctx lifetime, error strings, device status word and the
// Philox test aid.  The context plays the part of the per-worker state the
// reference keeps in Worker (src/worker.rs:13-38): the device it runs on and
// the stream its kernels go to.
#include <atomic>
#include <chrono>
#include <cstdlib>
#include <mutex>

#include "kyro_internal.cuh"
#include "kyro_math.h"

namespace kyro {

static thread_local std::string g_last_error;

int set_error(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_error(cudaError_t err, const char* what) {
  return set_error(KYRO_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, what);
  return KYRO_OK;
}

uint64_t default_wait_ns() {
  const char* e = std::getenv("KYRO_WAIT_TIMEOUT_MS");
  if (e && *e) {
    char* end = nullptr;
    const unsigned long v = std::strtoul(e, &end, 10);
    if (end && *end == '\0' && v >= 1 && v <= 600000) return (uint64_t)v * 1000000ull;
  }
  return 2000000000ull;  // 2 s
}

int enter(kyro_ctx* ctx) {
  if (!ctx) return set_error(KYRO_ERR_INVALID_ARG, "null kyro_ctx");
  cudaError_t err = cudaSetDevice(ctx->device);
  if (err != cudaSuccess) return cuda_error(err, "cudaSetDevice");
  return KYRO_OK;
}

}  // namespace kyro

namespace {

__global__ void philox_uniforms_kernel(uint64_t seed, uint32_t seq, uint32_t pos0,
                                       uint32_t stream, uint32_t step, int n, float* out) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n)
    out[i] = ky_odd_to_float(ky_uniform_odd(seed, seq, pos0 + (uint32_t)i, stream, step));
}

}  // namespace

extern "C" {

int kyro_version(void) { return KYRO_VERSION; }

const char* kyro_kernel_names(void) {
  return "accept_stats_kernel;accept_decide_kernel;accept_final_kernel;accept_tree_kernel;"
         "accept_tree_cluster_kernel;accept_tp_max_kernel;accept_tp_part_kernel;"
         "accept_tp_decide_kernel;accept_tp_search_kernel;accept_tp_write_kernel;"
         "verify_attention_kernel;kv_reserve_kernel;kv_commit_kernel;kv_commit_reserve_kernel;"
         "kv_tree_move_kernel;kv_write_kernel;rope_kv_write_kernel;kv_block_copy_kernel;"
         "philox_uniforms_kernel;exp_selftest_kernel;tree_attention_tc_kernel;peer_exchange_kernel";
}

size_t kyro_last_error(char* buf, size_t len) {
  const std::string& e = kyro::g_last_error;
  if (buf && len) {
    size_t n = e.size() < len - 1 ? e.size() : len - 1;
    memcpy(buf, e.data(), n);
    buf[n] = '\0';
  }
  return e.size();
}

const char* kyro_status_string(int status) {
  switch (status) {
    case KYRO_OK: return "ok";
    case KYRO_ERR_INVALID_ARG: return "invalid argument";
    case KYRO_ERR_CUDA: return "CUDA error";
    case KYRO_ERR_NCCL: return "NCCL error";
    case KYRO_ERR_TIMEOUT: return "timeout";
    case KYRO_ERR_OOB: return "out-of-bounds index detected on the device";
    case KYRO_ERR_OOM: return "out of KV blocks";
    case KYRO_ERR_UNSUPPORTED: return "unsupported configuration";
    case KYRO_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

int kyro_ctx_create(int device, void* stream, kyro_ctx** out) {
  if (!out) return kyro::set_error(KYRO_ERR_INVALID_ARG, "kyro_ctx_create: out is NULL");
  *out = nullptr;
  int count = 0;
  cudaError_t err = cudaGetDeviceCount(&count);
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaGetDeviceCount");
  if (device < 0 || device >= count)
    return kyro::set_error(KYRO_ERR_INVALID_ARG, "kyro_ctx_create: device %d of %d", device,
                           count);
  err = cudaSetDevice(device);
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaSetDevice");
  cudaDeviceProp prop;
  err = cudaGetDeviceProperties(&prop, device);
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return kyro::set_error(KYRO_ERR_UNSUPPORTED,
                           "kyro_ctx_create: device %d is sm_%d%d; this library is built for "
                           "sm_100a (B200) only",
                           device, prop.major, prop.minor);
  // the device may have been reset since an earlier context was made on it
  kyro::static_scratch_forget(device);
  kyro_ctx* ctx = new kyro_ctx();
  ctx->device = device;
  ctx->stream = (cudaStream_t)stream;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->nccl_comm = nullptr;
  ctx->tp_rank = 0;
  ctx->tp_world = 1;
  ctx->attn_epoch = 0;
  ctx->attn_ws_zeroed = nullptr;
  for (int i = 0; i < KYRO_ZEROED_WS; ++i) ctx->stats_ws_zeroed[i] = nullptr;
  ctx->stats_ws_next = 0;
  {
    // a salt per context: tags of different contexts differ
    static std::atomic<uint32_t> contexts{0};
    const uint64_t t = (uint64_t)std::chrono::steady_clock::now().time_since_epoch().count();
    ctx->pipe_salt = (uint32_t)(t ^ (t >> 32)) ^ (0x9E3779B9u * (contexts.fetch_add(1) + 1u));
  }
  ctx->xchg_ready = false;
  ctx->xchg_local = nullptr;
  for (int r = 0; r < KYRO_MAX_TP_WORLD; ++r) ctx->xchg_peer[r] = nullptr;
  ctx->xchg_skip_rounds = 0;
  ctx->wait_ns = kyro::default_wait_ns();
  ctx->watchdog = nullptr;
  ctx->tp_aborted = 0;
  // one allocation: the status word, then the acceptance pipeline's counts
  constexpr size_t kCtxBytes = 256 + 4 * KYRO_PIPE_COUNTS;
  err = cudaMalloc(&ctx->d_status, kCtxBytes);
  if (err != cudaSuccess) {
    delete ctx;
    return kyro::cuda_error(err, "cudaMalloc(status word)");
  }
  ctx->d_pipe_counts = ctx->d_status + 64;
  err = cudaMemset(ctx->d_status, 0, kCtxBytes);
  if (err != cudaSuccess) {
    cudaFree(ctx->d_status);
    delete ctx;
    return kyro::cuda_error(err, "cudaMemset(status word)");
  }
  *out = ctx;
  return KYRO_OK;
}

int kyro_ctx_destroy(kyro_ctx* ctx) {
  if (!ctx) return KYRO_OK;
  cudaSetDevice(ctx->device);
  kyro::nccl::release(ctx);
  cudaFree(ctx->d_status);
  delete ctx;
  return KYRO_OK;
}

int kyro_ctx_set_wait_timeout(kyro_ctx* ctx, uint32_t ms) {
  if (!ctx) return kyro::set_error(KYRO_ERR_INVALID_ARG, "null kyro_ctx");
  KY_REQUIRE(ms >= 1 && ms <= 600000, "kyro_ctx_set_wait_timeout: %u ms (1..600000)", ms);
  ctx->wait_ns = (uint64_t)ms * 1000000ull;
  return KYRO_OK;
}

int kyro_ctx_set_stream(kyro_ctx* ctx, void* stream) {
  if (!ctx) return kyro::set_error(KYRO_ERR_INVALID_ARG, "null kyro_ctx");
  ctx->stream = (cudaStream_t)stream;
  return KYRO_OK;
}

int kyro_ctx_device_status(kyro_ctx* ctx, uint32_t* out_flags, int clear) {
  KY_TRY(kyro::enter(ctx));
  cudaError_t err = cudaStreamSynchronize(ctx->stream);
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaStreamSynchronize");
  uint32_t flags = 0;
  err = cudaMemcpy(&flags, ctx->d_status, 4, cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return kyro::cuda_error(err, "read status word");
  if (clear) {
    err = cudaMemset(ctx->d_status, 0, 4);
    if (err != cudaSuccess) return kyro::cuda_error(err, "clear status word");
    // a wait that gave up may have left a call unfinished: move the
    // acceptance pipeline to a new generation (a new tag) with no sequence
    // counted
    if (flags & KYRO_DEV_WAIT_TIMEOUT) {
      uint32_t counts[2];
      err = cudaMemcpy(counts, ctx->d_pipe_counts, 8, cudaMemcpyDeviceToHost);
      if (err != cudaSuccess) return kyro::cuda_error(err, "read pipeline counts");
      counts[0] += 1u;
      counts[1] = 0u;
      err = cudaMemcpy(ctx->d_pipe_counts, counts, 8, cudaMemcpyHostToDevice);
      if (err != cudaSuccess) return kyro::cuda_error(err, "reset pipeline counts");
    }
  }
  if (out_flags) *out_flags = flags;
  return KYRO_OK;
}

int kyro_philox_uniforms(kyro_ctx* ctx, uint64_t seed, uint32_t seq, uint32_t pos0,
                         uint32_t stream, uint32_t step, int32_t n, float* out) {
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(n >= 0, "kyro_philox_uniforms: n = %d", n);
  KY_REQUIRE(n == 0 || out, "kyro_philox_uniforms: out is NULL");
  if (n == 0) return KYRO_OK;
  philox_uniforms_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>(seed, seq, pos0, stream, step,
                                                                   n, out);
  return kyro::check_launch("philox_uniforms_kernel");
}

}  // extern "C"
