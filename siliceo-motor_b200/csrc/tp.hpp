// Tensor parallelism of the decode path (Megatron split over one node's GPUs,
// one process per GPU): the exchange kernels that follow a row-split GEMV
// (all-reduce + residual + next RMSNorm input) and the vocab-split output
// head (all-gather of the logit slices), and the host side of a group.
//
// Exchanges run over peer memory: every rank owns a send arena and a flag
// array in its own HBM, mapped into every other rank (CUDA IPC over
// NVLink/NVSwitch). An exchange kernel block signals "my data is ready" into
// each peer's flag array with a system-scope release store, waits (bounded)
// for the peers' signals, then reads the peers' arenas with plain loads and
// combines them in rank order, so every rank computes bit-identical results.
// NCCL is used to form the group (unique id, IPC handle all-gather) and, with
// SM_TP_NCCL, as the collective itself.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace sm {

constexpr uint32_t TP_MAX = 8;
constexpr uint32_t TP_BLOCKS = 32;  // grid of every exchange kernel (flags and epochs are per block)

// Peer tables as the exchange kernels see them (passed by value).
struct TpPeers {
  uint32_t* flag[TP_MAX];  // rank r's flags [TP_BLOCKS][TP_MAX], mapped in this process
  uint32_t* epoch;         // this rank's per-block exchange counters [TP_BLOCKS]
  uint32_t* err;           // this rank's error word (bit TP_ERR_WAIT on a timed-out wait)
  uint64_t wait_ns;        // bound on one wait for a peer
  uint32_t rank, world;
  uint32_t sync;           // 0: sources are local (NCCL already exchanged), no flags
};
constexpr uint32_t TP_ERR_WAIT = 2u;

// x[r] += sum_k src[k][r] (k in rank order), xn[r] = x[r] * nw, and
// parts[r * TP_BLOCKS + block] = partial sums of x[r]^2 (the next GEMV's
// input-norm partials; n_parts = TP_BLOCKS). src rows have stride n.
cudaError_t launch_tp_reduce_resid(const TpPeers& p, const float* const* src, uint32_t nsrc, uint32_t rows, uint32_t n,
                                   float* x, uint32_t ldx, const float* nw, float* xn, uint32_t ldxn, float* parts,
                                   cudaStream_t st);
// out[r][k * nl + j] = src[k][r * nl + j] for j < min(nl, n_total - k * nl).
cudaError_t launch_tp_gather(const TpPeers& p, const float* const* src, uint32_t nsrc, uint32_t rows, uint32_t nl,
                             uint32_t n_total, float* out, uint32_t ldo, cudaStream_t st);

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
// id (bounded by wait_ms), the send arena of `arena_floats` floats per
// parity, and the peer mappings. Returns an sm_status; the message is set.
int tp_group_create(const void* id, uint32_t rank, uint32_t world, uint32_t flags, uint32_t wait_ms,
                    size_t arena_floats, size_t gather_floats, TpGroup** out);
// Waits (bounded) until every rank has reached this point: called by every
// rank once it makes no more exchanges, so that no peer still signals into
// an arena that is about to be freed.
void tp_group_barrier(TpGroup* g);
void tp_group_destroy(TpGroup* g);
// This rank's views for one exchange.
struct TpCall {
  TpPeers peers;
  const float* src[TP_MAX];
  uint32_t nsrc;
};
float* tp_send_buffer(TpGroup* g, uint32_t parity);  // local arena half the GEMV writes
float* tp_gather_buffer(TpGroup* g);                  // local slice the head GEMV writes
// Issues the collective part of an all-reduce of rows x n floats written to
// tp_send_buffer(parity) on stream st (NCCL mode), and returns the sources
// and peer tables for launch_tp_reduce_resid.
cudaError_t tp_allreduce_prepare(TpGroup* g, uint32_t parity, size_t count, cudaStream_t st, TpCall* call);
cudaError_t tp_gather_prepare(TpGroup* g, size_t count_per_rank, cudaStream_t st, TpCall* call);
bool tp_uses_nccl(const TpGroup* g);
int tp_unique_id(void* id_out);  // sm_status

}  // namespace sm
