// Expert-parallel prompt path: the routed-expert FFN of a MoE layer computed
// by the GPU that owns each expert, with the routed (token, rank) activation
// rows exchanged over NCCL (grouped point-to-point sends and receives, one
// process per GPU). See ep.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace lfm {

// Send plan of one MoE layer on one rank: slot j = token * 4 + rank of the
// routing sel[j] (expert id) goes to owner sel[j] / (32 / world). counts[o] =
// slots for owner o; order[i] = slot of send position i, owners ascending and
// slots ascending within an owner. Results come back in the same order, so the
// down row of slot order[i] is the i-th returned row.
void ep_plan(const int32_t* sel, int nslots, int world, int32_t* counts, int32_t* order);

// NCCL through the library the process already loaded (libnccl.so.2), so the
// engine and torch.distributed share one NCCL; false with a message if absent.
struct EpComm {
  void* comm = nullptr;  // ncclComm_t
  int rank = 0, world = 1;
};
bool ep_unique_id(uint8_t out[128], std::string& err);
bool ep_comm_init(EpComm& c, const uint8_t id[128], int rank, int world, std::string& err);
void ep_comm_destroy(EpComm& c);
// All ranks call these in the same order (one NCCL group each).
bool ep_allgather_i32(const EpComm& c, const int32_t* send, int32_t* recv, int count, cudaStream_t s,
                      std::string& err);
// Row exchange: rows of `width` floats (plus one int32 tag per row when tags
// are given): send_counts[p] rows from send + send_off[p] to p, recv_counts[p]
// rows from p into recv + recv_off[p].
bool ep_exchange(const EpComm& c, const float* send, const int32_t* send_tag, const int* send_counts,
                 const int* send_off, float* recv, int32_t* recv_tag, const int* recv_counts, const int* recv_off,
                 int width, cudaStream_t s, std::string& err);

// Device helpers.
// send[i] = rows[order[i] / 4] (the FFN input row of the slot's token), tag[i] = sel[order[i]].
void ep_pack(const float* rows, const int32_t* sel, const int32_t* order, int n, float* send, int32_t* tag,
             cudaStream_t s);
// Received slots as routing rows of 4 ranks for the grouped GEMMs: sel4[j] =
// tag[j] for j < n; the (at most 3) padding slots up to a multiple of 4 take
// the distinct experts pad, pad + 1, pad + 2 (local experts of this rank).
void ep_fake_sel(const int32_t* tag, int n, int pad, int32_t* sel4, cudaStream_t s);
// out[order[i]] = back[i] (rows of DIM floats).
void ep_unpack(const float* back, const int32_t* order, int n, float* out, cudaStream_t s);

}  // namespace lfm
