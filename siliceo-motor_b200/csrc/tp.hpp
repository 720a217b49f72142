// Tensor parallelism of the decode path (Megatron split over one node's GPUs,
// one process per GPU): the exchanges that follow a row-split GEMV
// (all-reduce + residual + next RMSNorm input) and the vocab-split output
// head (all-gather of the logit slices), and the host side of a group.
//
// Exchanges are pushes over peer memory: every rank owns receive areas in its
// own HBM, mapped into every other rank (CUDA IPC over NVLink/NVSwitch). The
// producing GEMV's epilogue (EPI_PUSH, device.cuh) stores each output as an
// 8-byte packet (value | epoch) into every rank's area, so the data and its
// "ready" mark cross NVLink in one write, without fences or flags; the
// consumer kernel polls its local packets (bounded) until they carry the
// exchange's epoch, then combines the ranks in rank order, so every rank
// computes bit-identical results. NCCL forms the group (unique id, IPC handle
// all-gather) and, with SM_TP_NCCL, is the collective itself.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "device.cuh"

namespace sm {

constexpr uint32_t TP_MAX = TP_MAX_RANKS;
constexpr uint32_t TP_BLOCKS = 32;  // consumer blocks per exchange (epochs are per block)
constexpr uint32_t TP_ERR_WAIT = 2u;

// A receive area as its consumer kernel sees it.
struct TpRecv {
  const uint64_t* pk;      // packets [parity][source rank][row][ld] (parity_stride 0: one half)
  const float* plain;      // instead of packets (NCCL mode): f32 data already exchanged
  uint64_t parity_stride;  // packets between the halves
  uint64_t src_stride;     // packets (or floats of `plain`) between source ranks
  uint32_t* epoch;         // this rank's per-block epochs of this exchange kind
  uint32_t* err;           // this rank's error word (TP_ERR_WAIT on a timed-out wait)
  uint64_t wait_ns;        // bound on one wait
  uint32_t world, ld, per; // per: elements of a consumer block
};

// x[r][o] += sum over ranks k (in order) of their partials, xn = x * nw, and
// parts[r * TP_BLOCKS + block] = partial sums of x[r]^2 (the next GEMV's
// input-norm partials; n_parts = TP_BLOCKS).
cudaError_t launch_tp_reduce_resid(const TpRecv& rv, uint32_t rows, uint32_t n, float* x, uint32_t ldx, const float* nw,
                                   float* xn, uint32_t ldxn, float* parts, cudaStream_t st);
// out[r][v] for v < n_total: the slice of rank v / nl at v % nl.
cudaError_t launch_tp_gather(const TpRecv& rv, uint32_t rows, uint32_t nl, uint32_t n_total, float* out, uint32_t ldo,
                             cudaStream_t st);

// ------------------------------------------------------------ host side ----
// How each rank splits a model (column split = output rows, row split =
// input columns of a weight).
struct TpShard {
  uint32_t rank = 0, world = 1;
  uint64_t q_heads = 0, kv_heads = 0;  // local heads (first: rank * count)
  uint64_t ff = 0;                     // local FFN width (first: rank * ff)
  uint64_t vocab = 0, vocab0 = 0;      // local output-head rows [vocab0, vocab0 + vocab)
  uint64_t vocab_stride = 0;           // rows per rank (the last rank may have fewer)
};
// Returns "" if the model can be split this way, else the reason.
std::string tp_plan(uint64_t n_heads, uint64_t n_kv_heads, uint64_t head_dim, uint64_t n_ff, uint64_t vocab,
                    uint32_t block_in_o, uint32_t block_in_down, uint32_t rank, uint32_t world, TpShard* out);

struct TpGroup;
// Forms the group on the current device: NCCL communicator from the shared
// id (bounded by wait_ms), receive areas for all-reduces of rows x n floats
// and gathers of rows x nl floats per rank, and the peer mappings. Returns an
// sm_status; the message is set.
int tp_group_create(const void* id, uint32_t rank, uint32_t world, uint32_t flags, uint32_t wait_ms, uint32_t rows,
                    uint32_t n, uint32_t nl, TpGroup** out);
// Waits (bounded) until every rank has reached this point: called by every
// rank once it makes no more exchanges, so that no peer still writes into
// an area that is about to be freed.
void tp_group_barrier(TpGroup* g);
void tp_group_destroy(TpGroup* g);
bool tp_uses_nccl(const TpGroup* g);
int tp_unique_id(void* id_out);  // sm_status

// One all-reduce / gather. The producing GEMV gets either `push` (EPI_PUSH,
// peer-memory mode) or writes `send` with EPI_STORE (NCCL mode; tp_*_issue
// then runs the collective); the consumer kernel gets `recv`.
struct TpExchange {
  TpPush push;
  float* send;
  TpRecv recv;
};
TpExchange tp_allreduce(TpGroup* g, uint32_t* err);
TpExchange tp_gather(TpGroup* g, uint32_t rows, uint64_t vocab0, uint32_t* err);
cudaError_t tp_allreduce_issue(TpGroup* g, uint32_t rows, cudaStream_t st);
cudaError_t tp_gather_issue(TpGroup* g, uint32_t rows, cudaStream_t st);

}  // namespace sm
