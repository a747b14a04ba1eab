// The library's context and the host-side helpers its C-ABI entry points share (internal:
// included by g4_abi.cu and g4_decoder.cu only).
#pragma once

#include <cstdio>
#include <initializer_list>
#include <utility>

#include "../../include/g4b200.h"
#include "g4_ops.cuh"

namespace g4 {
int attention_slot_multiple();
int attention_max_ring();
}  // namespace g4

struct g4_ctx {
  int device = 0;
  int sm_count = 0;
  bool overlap = false;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  g4::Scratch sc{};
  size_t act_bytes = 0;
  bool batch_ok = false;  // the batched feed-forward's launch geometry fits this GPU
  g4::TmapCache maps;
  // tensor parallelism (g4_tp_init / g4_tp_connect); world 1 until then
  int tp_rank = 0, tp_world = 1;
  bool tp_ready = true;                    // connected (a world of 1 needs no peers)
  void* tp_buf = nullptr;                  // this rank's exchange buffer, then its epoch counters
  void* tp_peer[g4::kMaxTp] = {};          // the peers' buffers, opened in this process
  unsigned char tp_blob[G4_TP_BLOB_BYTES] = {0};
  uint32_t tp_generation = 0;              // setups of the group so far (agreed at connect)
  uint64_t tp_wait_ns = g4::kWaitLimitNs;  // limit of the exchange's wait for the peers
  g4::TpLink tp{0, 1, {}, nullptr, 0, g4::kWaitLimitNs};
  char last_error[256] = {0};
};

namespace g4::host {

// Restores the caller's current device when the call returns.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

inline g4_status fail(g4_ctx* ctx, g4_status st, const char* fmt, const char* what) {
  if (ctx) snprintf(ctx->last_error, sizeof ctx->last_error, fmt, what);
  return st;
}

inline g4_status cuda_status(g4_ctx* ctx, cudaError_t e, const char* where) {
  if (e == cudaSuccess) return G4_OK;
  if (ctx) snprintf(ctx->last_error, sizeof ctx->last_error, "%s: %s", where, cudaGetErrorString(e));
  return G4_ERR_CUDA;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Every pointer non-null and 16-byte aligned.
inline g4_status check_ptrs(g4_ctx* ctx, std::initializer_list<std::pair<const void*, const char*>> ptrs) {
  for (const auto& p : ptrs) {
    if (!p.first) return fail(ctx, G4_ERR_INVALID_ARGUMENT, "null pointer: %s", p.second);
    if (!aligned16(p.first)) return fail(ctx, G4_ERR_MISALIGNED, "pointer not 16-byte aligned: %s", p.second);
  }
  return G4_OK;
}

inline g4::LaunchEnv env_of(g4_ctx* ctx, void* stream) {
  g4::LaunchEnv env;
  env.device = ctx->device;
  env.sm_count = ctx->sm_count;
  env.stream = static_cast<cudaStream_t>(stream);
  env.pdl = ctx->overlap;
  env.sc = ctx->sc;
  env.maps = &ctx->maps;
  env.tp = ctx->tp;
  return env;
}

// Ops of a tensor-parallel context run only once it is connected to its peers.
inline g4_status check_tp(g4_ctx* ctx) {
  if (ctx->tp_ready) return G4_OK;
  return fail(ctx, G4_ERR_INVALID_ARGUMENT, "%s", "tensor-parallel context is not connected (g4_tp_connect)");
}

}  // namespace g4::host
