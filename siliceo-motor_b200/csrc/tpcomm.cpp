// Host side of a tensor-parallel group (see tp.hpp): the split plan, the
// NCCL communicator that forms the group, and the peer-memory arenas the
// exchange kernels use.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the library the
// process already has if PyTorch loaded one), so the engine has no link-time
// dependency on it and single-GPU use never touches it. Every blocking step
// of group formation is bounded: the communicator is created non-blocking
// and polled against a deadline, and a timed-out group is aborted.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "../../include/sm_engine.h"
#include "common.hpp"
#include "tp.hpp"

namespace sm {
namespace {

struct NcclApi {
  void* h = nullptr;
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) get_async_error = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  std::string why;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    api.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!api.h) {
      const char* e = dlerror();
      api.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "?");
      return;
    }
    bool ok = true;
    auto sym = [&](auto& f, const char* name) {
      f = reinterpret_cast<std::remove_reference_t<decltype(f)>>(dlsym(api.h, name));
      ok &= f != nullptr;
    };
    sym(api.get_unique_id, "ncclGetUniqueId");
    sym(api.init_rank_config, "ncclCommInitRankConfig");
    sym(api.get_async_error, "ncclCommGetAsyncError");
    sym(api.abort, "ncclCommAbort");
    sym(api.destroy, "ncclCommDestroy");
    sym(api.all_reduce, "ncclAllReduce");
    sym(api.all_gather, "ncclAllGather");
    sym(api.error_string, "ncclGetErrorString");
    if (!ok) {
      api.why = "libnccl.so.2 lacks a needed symbol";
      api.h = nullptr;
    }
  });
  return api;
}

using Clock = std::chrono::steady_clock;

}  // namespace

// This rank's arena (one allocation, mapped by every peer):
//   epochs: all-reduce [TP_BLOCKS] | gather [TP_BLOCKS]
//   all-reduce packets [2 halves][world sources][rows][n]
//   gather packets [world sources][rows][nl]
//   NCCL mode: send f32 [rows][n] | receive f32 [rows][n] | gather send f32 [rows][nl] | gather receive [world][rows][nl]
struct TpGroup {
  uint32_t rank = 0, world = 1, flags = 0, rows = 0, n = 0, nl = 0;
  uint64_t wait_ns = 0;
  ncclComm_t comm = nullptr;
  uint8_t* arena = nullptr;
  uint8_t* peer[TP_MAX] = {};
  size_t off_ep_ar = 0, off_ep_g = 0, off_ar = 0, off_g = 0, off_send = 0, off_recv = 0, off_gsend = 0, off_grecv = 0;
  bool opened[TP_MAX] = {};
};

namespace {

std::string nccl_text(ncclResult_t r) {
  const NcclApi& a = nccl();
  return a.error_string ? a.error_string(r) : ("NCCL error " + std::to_string((int)r));
}

// Waits until the communicator's pending work is enqueued (non-blocking
// communicators return ncclInProgress), bounded by the deadline.
int nccl_settle(TpGroup* g, ncclResult_t rc, Clock::time_point deadline, const char* what) {
  const NcclApi& a = nccl();
  while (rc == ncclInProgress) {
    if (Clock::now() > deadline) {
      set_error(std::string("tensor-parallel group: ") + what + " did not complete in time (a rank is missing)");
      return SM_ERR_PEER;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
    ncclResult_t st = ncclInProgress;
    if (a.get_async_error(g->comm, &st) != ncclSuccess) st = ncclSystemError;
    rc = st;
  }
  if (rc != ncclSuccess) {
    set_error(std::string("tensor-parallel group: ") + what + ": " + nccl_text(rc));
    return SM_ERR_PEER;
  }
  return SM_OK;
}

// Waits for the stream's work (bounded): a collective whose peer never comes
// never completes.
int stream_settle(TpGroup* g, cudaStream_t st, Clock::time_point deadline, const char* what) {
  for (;;) {
    cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return SM_OK;
    if (e != cudaErrorNotReady) {
      set_error(std::string("tensor-parallel group: ") + what + ": " + cudaGetErrorString(e));
      return SM_ERR_CUDA;
    }
    if (Clock::now() > deadline) {
      set_error(std::string("tensor-parallel group: ") + what + " did not complete in time (a rank is missing)");
      return SM_ERR_PEER;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

size_t up256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

std::string tp_plan(uint64_t n_heads, uint64_t n_kv_heads, uint64_t head_dim, uint64_t n_ff, uint64_t vocab,
                    uint32_t block_in_o, uint32_t block_in_down, uint32_t rank, uint32_t world, TpShard* out) {
  if (world < 1 || world > TP_MAX) return "tensor-parallel size must be 1.." + std::to_string(TP_MAX);
  if (rank >= world) return "tensor-parallel rank must be below the size";
  if (n_kv_heads % world) return "kv heads (" + std::to_string(n_kv_heads) + ") do not divide by the tensor-parallel size";
  if (n_heads % world) return "query heads do not divide by the tensor-parallel size";
  if (n_ff % world) return "the FFN width does not divide by the tensor-parallel size";
  const uint64_t qd = n_heads / world * head_dim, ff = n_ff / world;
  if (block_in_o && qd % block_in_o)
    return "attn_output's split input (" + std::to_string(qd) + ") is not a whole number of quant blocks";
  if (block_in_down && ff % block_in_down)
    return "ffn_down's split input (" + std::to_string(ff) + ") is not a whole number of quant blocks";
  TpShard s;
  s.rank = rank;
  s.world = world;
  s.q_heads = n_heads / world;
  s.kv_heads = n_kv_heads / world;
  s.ff = ff;
  s.vocab_stride = (vocab + world - 1) / world;
  s.vocab0 = std::min<uint64_t>(vocab, (uint64_t)rank * s.vocab_stride);
  s.vocab = std::min<uint64_t>(vocab, s.vocab0 + s.vocab_stride) - s.vocab0;
  if (s.vocab == 0) return "the vocabulary is too small for this tensor-parallel size";
  *out = s;
  return "";
}

int tp_unique_id(void* id_out) {
  const NcclApi& a = nccl();
  if (!a.h) { set_error(a.why); return SM_ERR_UNSUPPORTED; }
  ncclUniqueId id;
  ncclResult_t r = a.get_unique_id(&id);
  if (r != ncclSuccess) { set_error("ncclGetUniqueId: " + nccl_text(r)); return SM_ERR_PEER; }
  static_assert(sizeof(ncclUniqueId) == SM_TP_ID_BYTES, "NCCL unique id size");
  std::memcpy(id_out, &id, sizeof id);
  return SM_OK;
}

void tp_group_barrier(TpGroup* g) {
  const NcclApi& a = nccl();
  if (!g || !g->comm || !g->arena || !a.h) return;
  cudaStream_t st = nullptr;
  if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess) {
    const auto deadline = Clock::now() + std::chrono::nanoseconds(g->wait_ns);
    // a scratch float of the arena that no exchange uses any more
    float* b = reinterpret_cast<float*>(g->arena + (tp_uses_nccl(g) ? g->off_send : g->off_ar));
    ncclResult_t r = a.all_reduce(b, b, 1, ncclFloat, ncclSum, g->comm, st);
    if (nccl_settle(g, r, deadline, "teardown barrier") == SM_OK) stream_settle(g, st, deadline, "teardown barrier");
    cudaStreamDestroy(st);
  }
  cudaGetLastError();
}

void tp_group_destroy(TpGroup* g) {
  if (!g) return;
  const NcclApi& a = nccl();
  for (uint32_t r = 0; r < TP_MAX; r++)
    if (g->opened[r]) cudaIpcCloseMemHandle(g->peer[r]);
  if (g->comm && a.h) {
    // A group whose formation or exchanges failed may have work in flight
    // that never completes: abort it instead of waiting.
    a.abort(g->comm);
  }
  if (g->arena) cudaFree(g->arena);
  delete g;
}


int tp_group_create(const void* id, uint32_t rank, uint32_t world, uint32_t flags, uint32_t wait_ms, uint32_t rows,
                    uint32_t n, uint32_t nl, TpGroup** out) {
  const NcclApi& a = nccl();
  if (!a.h) { set_error(a.why); return SM_ERR_UNSUPPORTED; }
  if (!id || world < 2 || world > TP_MAX || rank >= world || !rows || !n || !nl) {
    set_error("tensor-parallel group: bad rank/size/id");
    return SM_ERR_ARG;
  }
  auto* g = new TpGroup();
  g->rank = rank;
  g->world = world;
  g->flags = flags;
  g->rows = rows;
  g->n = n;
  g->nl = nl;
  g->wait_ns = (uint64_t)(wait_ms ? wait_ms : 10000u) * 1000000ull;
  const auto deadline = Clock::now() + std::chrono::milliseconds(wait_ms ? wait_ms : 10000u) * 6;
  int rc = SM_OK;
  cudaStream_t st = nullptr;
  auto fail = [&](int code) {
    if (st) cudaStreamDestroy(st);
    const std::string msg = get_error();
    tp_group_destroy(g);
    set_error(msg);
    return code;
  };
  // 1. communicator (non-blocking, polled against the deadline)
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof uid);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = a.init_rank_config(&g->comm, (int)world, uid, (int)rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    set_error("tensor-parallel group: ncclCommInitRankConfig: " + nccl_text(r));
    g->comm = nullptr;
    return fail(SM_ERR_PEER);
  }
  if ((rc = nccl_settle(g, r, deadline, "communicator set-up"))) return fail(rc);
  // 2. arena (zeroed: every epoch 0, no packet carries an exchange's epoch)
  const bool use_nccl = flags & SM_TP_NCCL;
  const size_t rn = (size_t)rows * n, rl = (size_t)rows * nl;
  size_t off = 0;
  g->off_ep_ar = off; off += up256(TP_BLOCKS * 4);
  g->off_ep_g = off; off += up256(TP_BLOCKS * 4);
  g->off_ar = off; off += up256(2 * world * rn * 8);
  g->off_g = off; off += up256(world * rl * 8);
  if (use_nccl) {
    g->off_send = off; off += up256(rn * 4);
    g->off_recv = off; off += up256(rn * 4);
    g->off_gsend = off; off += up256(rl * 4);
    g->off_grecv = off; off += up256(world * rl * 4);
  }
  if (cudaMalloc(&g->arena, off) != cudaSuccess) {
    cudaGetLastError();
    set_error("tensor-parallel group: cudaMalloc of the exchange arena failed");
    return fail(SM_ERR_OOM);
  }
  if (cudaMemset(g->arena, 0, off) != cudaSuccess || cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    set_error("tensor-parallel group: arena set-up failed");
    return fail(SM_ERR_CUDA);
  }
  // 3. exchange the arenas' IPC handles (NCCL all-gather) and map the peers'
  cudaIpcMemHandle_t mine;
  if (cudaIpcGetMemHandle(&mine, g->arena) != cudaSuccess) {
    cudaGetLastError();
    set_error("tensor-parallel group: cudaIpcGetMemHandle failed");
    return fail(SM_ERR_CUDA);
  }
  uint8_t* dh = nullptr;
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  if (cudaMalloc(&dh, hb * world) != cudaSuccess ||
      cudaMemcpy(dh + hb * rank, &mine, hb, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    if (dh) cudaFree(dh);
    set_error("tensor-parallel group: handle buffer failed");
    return fail(SM_ERR_CUDA);
  }
  r = a.all_gather(dh + hb * rank, dh, hb, ncclChar, g->comm, st);
  if ((rc = nccl_settle(g, r, deadline, "handle exchange")) || (rc = stream_settle(g, st, deadline, "handle exchange"))) {
    cudaFree(dh);
    return fail(rc);
  }
  std::vector<cudaIpcMemHandle_t> all(world);
  cudaError_t ce = cudaMemcpy(all.data(), dh, hb * world, cudaMemcpyDeviceToHost);
  cudaFree(dh);
  if (ce != cudaSuccess) { set_error("tensor-parallel group: handle copy failed"); return fail(SM_ERR_CUDA); }
  for (uint32_t k = 0; k < world; k++) {
    if (k == rank) { g->peer[k] = g->arena; continue; }
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[k], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      set_error("tensor-parallel group: cannot map rank " + std::to_string(k) +
                "'s memory (peer access over NVLink is required)");
      return fail(SM_ERR_PEER);
    }
    g->peer[k] = (uint8_t*)p;
    g->opened[k] = true;
  }
  // 4. warm the collectives up outside any graph capture; this also makes
  //    every rank map its peers before any of them pushes.
  {
    float* b = reinterpret_cast<float*>(g->arena + (use_nccl ? g->off_send : g->off_ar));
    r = a.all_reduce(b, b, 64, ncclFloat, ncclSum, g->comm, st);
    if ((rc = nccl_settle(g, r, deadline, "warm-up all-reduce")) || (rc = stream_settle(g, st, deadline, "warm-up all-reduce")))
      return fail(rc);
    if (use_nccl) {
      r = a.all_gather(reinterpret_cast<float*>(g->arena + g->off_gsend),
                       reinterpret_cast<float*>(g->arena + g->off_grecv), std::min<size_t>(rl, 64), ncclFloat, g->comm,
                       st);
      if ((rc = nccl_settle(g, r, deadline, "warm-up all-gather")) || (rc = stream_settle(g, st, deadline, "warm-up all-gather")))
        return fail(rc);
    }
    if (cudaMemsetAsync(b, 0, 64 * 4, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) {
      cudaGetLastError();
      set_error("tensor-parallel group: warm-up failed");
      return fail(SM_ERR_CUDA);
    }
  }
  cudaStreamDestroy(st);
  *out = g;
  return SM_OK;
}

bool tp_uses_nccl(const TpGroup* g) { return g->flags & SM_TP_NCCL; }

namespace {
TpRecv recv_base(TpGroup* g, uint32_t* err) {
  TpRecv r{};
  r.err = err;
  r.wait_ns = g->wait_ns;
  r.world = g->world;
  return r;
}

cudaError_t nccl_issue(TpGroup* g, ncclResult_t r) {
  if (r == ncclInProgress &&
      nccl_settle(g, r, Clock::now() + std::chrono::nanoseconds(g->wait_ns), "collective") != SM_OK)
    return cudaErrorLaunchFailure;
  return (r == ncclSuccess || r == ncclInProgress) ? cudaSuccess : cudaErrorLaunchFailure;
}
}  // namespace

TpExchange tp_allreduce(TpGroup* g, uint32_t* err) {
  TpExchange x{};
  x.recv = recv_base(g, err);
  x.recv.ld = g->n;
  x.recv.per = (g->n + TP_BLOCKS - 1) / TP_BLOCKS;
  if (tp_uses_nccl(g)) {
    x.send = reinterpret_cast<float*>(g->arena + g->off_send);
    x.recv.plain = reinterpret_cast<const float*>(g->arena + g->off_recv);
    return x;
  }
  const uint64_t rn = (uint64_t)g->rows * g->n;
  for (uint32_t k = 0; k < g->world; k++) x.push.dst[k] = reinterpret_cast<uint64_t*>(g->peer[k] + g->off_ar);
  x.push.parity_stride = g->world * rn;
  x.push.src_stride = rn;
  x.push.epoch = reinterpret_cast<const uint32_t*>(g->arena + g->off_ep_ar);
  x.push.world = g->world;
  x.push.rank = g->rank;
  x.push.ld = g->n;
  x.push.per = x.recv.per;
  x.push.base = 0;
  x.recv.pk = reinterpret_cast<const uint64_t*>(g->arena + g->off_ar);
  x.recv.parity_stride = x.push.parity_stride;
  x.recv.src_stride = rn;
  x.recv.epoch = reinterpret_cast<uint32_t*>(g->arena + g->off_ep_ar);
  return x;
}

TpExchange tp_gather(TpGroup* g, uint32_t rows, uint64_t vocab0, uint32_t* err) {
  TpExchange x{};
  x.recv = recv_base(g, err);
  x.recv.ld = g->nl;
  const uint64_t total = (uint64_t)g->nl * g->world;
  x.recv.per = (uint32_t)((total + TP_BLOCKS - 1) / TP_BLOCKS);
  if (tp_uses_nccl(g)) {
    x.send = reinterpret_cast<float*>(g->arena + g->off_gsend);
    x.recv.plain = reinterpret_cast<const float*>(g->arena + g->off_grecv);
    x.recv.src_stride = (uint64_t)rows * g->nl;  // all-gather output: [rank][rows][nl]
    return x;
  }
  const uint64_t rl = (uint64_t)g->rows * g->nl;
  for (uint32_t k = 0; k < g->world; k++) x.push.dst[k] = reinterpret_cast<uint64_t*>(g->peer[k] + g->off_g);
  x.push.parity_stride = 0;
  x.push.src_stride = rl;
  x.push.epoch = reinterpret_cast<const uint32_t*>(g->arena + g->off_ep_g);
  x.push.world = g->world;
  x.push.rank = g->rank;
  x.push.ld = g->nl;
  x.push.per = x.recv.per;
  x.push.base = (uint32_t)vocab0;
  x.recv.pk = reinterpret_cast<const uint64_t*>(g->arena + g->off_g);
  x.recv.src_stride = rl;
  x.recv.epoch = reinterpret_cast<uint32_t*>(g->arena + g->off_ep_g);
  return x;
}

cudaError_t tp_allreduce_issue(TpGroup* g, uint32_t rows, cudaStream_t st) {
  return nccl_issue(g, nccl().all_reduce(g->arena + g->off_send, g->arena + g->off_recv, (size_t)rows * g->n, ncclFloat,
                                         ncclSum, g->comm, st));
}

cudaError_t tp_gather_issue(TpGroup* g, uint32_t rows, cudaStream_t st) {
  return nccl_issue(g, nccl().all_gather(g->arena + g->off_gsend, g->arena + g->off_grecv, (size_t)rows * g->nl,
                                         ncclFloat, g->comm, st));
}

}  // namespace sm
