// A C++ caller of libkyro_spec through include/kyro_spec.h alone (no
// ctypes, no torch): the way a native host such as a Rust worker binds the
// library.  It reads one acceptance case from a file, runs kyro_spec_accept
// on device 0 and writes the outputs.
//
//   accept_harness <in.bin> <out.bin>   run the case
//   accept_harness --no-gpu             check the host-side error path on a
//                                       machine without a GPU
//
// in.bin:  int32 B, k, V, mode; float T; uint32 step; uint64 seed;
//          float target[B][k+1][V]; float draft[B][k][V]; int32 drafts[B][k]
// out.bin: int32 accept_len[B]; int32 tokens[B][k+1]; int32 num[B];
//          float probs[B][k][2]; uint32 device status
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "kyro_spec.h"

static int fail(const char* what, int st) {
  char msg[512];
  kyro_last_error(msg, sizeof msg);
  std::fprintf(stderr, "%s: %s (%s)\n", what, kyro_status_string(st), msg);
  return 1;
}

static int no_gpu() {
  // the library loads and answers without a device; creating a context
  // fails cleanly with a message, and null arguments are rejected
  if (kyro_version() != KYRO_VERSION) return 2;
  kyro_ctx* ctx = nullptr;
  const int st = kyro_ctx_create(0, nullptr, &ctx);
  if (st == KYRO_OK || ctx != nullptr) return 3;
  char msg[512];
  if (kyro_last_error(msg, sizeof msg) == 0) return 4;
  kyro_accept_params p = {8, 4, 32000, KYRO_ACCEPT_STOCHASTIC, 1.0f, 0, 0, 0};
  if (kyro_spec_accept(nullptr, &p, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                       nullptr, nullptr, 0) != KYRO_ERR_INVALID_ARG)
    return 5;
  if (kyro_spec_accept_workspace_size(&p) == 0) return 6;
  std::printf("no-gpu ok: %s\n", msg);
  return 0;
}

int main(int argc, char** argv) {
  if (argc == 2 && std::strcmp(argv[1], "--no-gpu") == 0) return no_gpu();
  if (argc != 3) {
    std::fprintf(stderr, "usage: %s <in.bin> <out.bin> | --no-gpu\n", argv[0]);
    return 64;
  }
  FILE* f = std::fopen(argv[1], "rb");
  if (!f) return 65;
  int32_t hdr[4];
  float T;
  uint32_t step;
  uint64_t seed;
  if (std::fread(hdr, 4, 4, f) != 4 || std::fread(&T, 4, 1, f) != 1 ||
      std::fread(&step, 4, 1, f) != 1 || std::fread(&seed, 8, 1, f) != 1)
    return 66;
  const int B = hdr[0], k = hdr[1], V = hdr[2], mode = hdr[3];
  std::vector<float> tgt((size_t)B * (k + 1) * V), drf((size_t)B * k * V);
  std::vector<int32_t> drafts((size_t)B * k);
  if (std::fread(tgt.data(), 4, tgt.size(), f) != tgt.size() ||
      std::fread(drf.data(), 4, drf.size(), f) != drf.size() ||
      std::fread(drafts.data(), 4, drafts.size(), f) != drafts.size())
    return 67;
  std::fclose(f);

  kyro_ctx* ctx = nullptr;
  int st = kyro_ctx_create(0, nullptr, &ctx);
  if (st != KYRO_OK) return fail("kyro_ctx_create", st);
  kyro_accept_params p = {B, k, V, mode, T, step, seed, 0};
  const size_t ws_bytes = kyro_spec_accept_workspace_size(&p);
  float *d_tgt, *d_drf, *d_probs;
  int32_t *d_drafts, *d_acc, *d_toks, *d_num;
  void* d_ws;
  cudaMalloc(&d_tgt, tgt.size() * 4);
  cudaMalloc(&d_drf, drf.size() * 4 + 4);
  cudaMalloc(&d_drafts, drafts.size() * 4 + 4);
  cudaMalloc(&d_acc, (size_t)B * 4);
  cudaMalloc(&d_toks, (size_t)B * (k + 1) * 4);
  cudaMalloc(&d_num, (size_t)B * 4);
  cudaMalloc(&d_probs, (size_t)B * k * 2 * 4 + 4);
  cudaMalloc(&d_ws, ws_bytes);
  if (cudaGetLastError() != cudaSuccess) return 68;
  cudaMemcpy(d_tgt, tgt.data(), tgt.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(d_drf, drf.data(), drf.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(d_drafts, drafts.data(), drafts.size() * 4, cudaMemcpyHostToDevice);
  st = kyro_spec_accept(ctx, &p, d_tgt, mode == KYRO_ACCEPT_STOCHASTIC ? d_drf : nullptr,
                        d_drafts, d_acc, d_toks, d_num, d_probs, d_ws, ws_bytes);
  if (st != KYRO_OK) return fail("kyro_spec_accept", st);
  uint32_t flags = 0;
  st = kyro_ctx_device_status(ctx, &flags, 1);
  if (st != KYRO_OK) return fail("kyro_ctx_device_status", st);
  std::vector<int32_t> acc(B), toks((size_t)B * (k + 1)), num(B);
  std::vector<float> probs((size_t)B * k * 2);
  cudaMemcpy(acc.data(), d_acc, acc.size() * 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(toks.data(), d_toks, toks.size() * 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(num.data(), d_num, num.size() * 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(probs.data(), d_probs, probs.size() * 4, cudaMemcpyDeviceToHost);
  FILE* o = std::fopen(argv[2], "wb");
  if (!o) return 69;
  std::fwrite(acc.data(), 4, acc.size(), o);
  std::fwrite(toks.data(), 4, toks.size(), o);
  std::fwrite(num.data(), 4, num.size(), o);
  std::fwrite(probs.data(), 4, probs.size(), o);
  std::fwrite(&flags, 4, 1, o);
  std::fclose(o);
  for (void* ptr : {(void*)d_tgt, (void*)d_drf, (void*)d_drafts, (void*)d_acc, (void*)d_toks,
                    (void*)d_num, (void*)d_probs, d_ws})
    cudaFree(ptr);
  kyro_ctx_destroy(ctx);
  return 0;
}
