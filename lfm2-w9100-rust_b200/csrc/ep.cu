// Expert-parallel prompt path (see ep.h): the send plan, the NCCL row
// exchange and the pack / unpack kernels around it.
//
// Placement: expert e lives on rank e / (32 / world) (world = 2, 4 or 8). A
// MoE layer on each rank: route its own tokens, send every routed
// (token, rank) slot's FFN input row to the expert's owner, run the owner's
// grouped gate/up -> SwiGLU -> down GEMMs on the slots it received, send the
// down rows back in the order they came, and combine them in rank order
// (kernels/resident.rs:101-117), so the result equals the single-GPU layer's.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <type_traits>

#include "ep.h"
#include "kernels.h"

namespace lfm {

void ep_plan(const int32_t* sel, int nslots, int world, int32_t* counts, int32_t* order) {
  const int per = N_EXPERT / world;
  std::vector<int32_t> start(world + 1, 0);
  for (int o = 0; o < world; o++) counts[o] = 0;
  for (int j = 0; j < nslots; j++) counts[sel[j] / per]++;
  for (int o = 0; o < world; o++) start[o + 1] = start[o] + counts[o];
  for (int j = 0; j < nslots; j++) order[start[sel[j] / per]++] = j;  // stable: slots ascending per owner
}

namespace {
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  std::string why;
};

// libnccl.so.2 by its soname: the copy torch.distributed already loaded when
// there is one, else the system library.
const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.why = std::string("libnccl.so.2 not found: ") + dlerror();
      return;
    }
    auto sym = [&](const char* name, auto& fn) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    api.ok = sym("ncclGetUniqueId", api.get_unique_id) && sym("ncclCommInitRank", api.comm_init_rank) &&
             sym("ncclCommDestroy", api.comm_destroy) && sym("ncclGroupStart", api.group_start) &&
             sym("ncclGroupEnd", api.group_end) && sym("ncclSend", api.send) && sym("ncclRecv", api.recv) &&
             sym("ncclAllGather", api.all_gather) && sym("ncclGetErrorString", api.error_string);
    if (!api.ok) api.why = "libnccl.so.2 lacks a required entry point";
  });
  return api;
}

bool nccl_ok(ncclResult_t r, const char* what, std::string& err) {
  if (r == ncclSuccess) return true;
  err = std::string(what) + ": " + nccl().error_string(r);
  return false;
}

__global__ void k_ep_pack(const float* rows, const int32_t* sel, const int32_t* order, int n, float* send,
                          int32_t* tag) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const int j = order[i];
  const float4* src = (const float4*)(rows + (size_t)(j / N_USED) * DIM);
  float4* dst = (float4*)(send + (size_t)i * DIM);
  for (int c = threadIdx.x; c < DIM / 4; c += blockDim.x) dst[c] = src[c];
  if (threadIdx.x == 0) tag[i] = sel[j];
}

__global__ void k_ep_fake_sel(const int32_t* tag, int n, int pad, int32_t* sel4) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  const int n4 = (n + N_USED - 1) / N_USED * N_USED;
  if (j < n4) sel4[j] = j < n ? tag[j] : pad + (j - n);  // at most 3 padding slots, distinct experts
}

__global__ void k_ep_unpack(const float* back, const int32_t* order, int n, float* out) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const float4* src = (const float4*)(back + (size_t)i * DIM);
  float4* dst = (float4*)(out + (size_t)order[i] * DIM);
  for (int c = threadIdx.x; c < DIM / 4; c += blockDim.x) dst[c] = src[c];
}
}  // namespace

bool ep_unique_id(uint8_t out[128], std::string& err) {
  const NcclApi& a = nccl();
  if (!a.ok) {
    err = a.why;
    return false;
  }
  ncclUniqueId id;
  if (!nccl_ok(a.get_unique_id(&id), "ncclGetUniqueId", err)) return false;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  memcpy(out, &id, 128);
  return true;
}

bool ep_comm_init(EpComm& c, const uint8_t id[128], int rank, int world, std::string& err) {
  const NcclApi& a = nccl();
  if (!a.ok) {
    err = a.why;
    return false;
  }
  ncclUniqueId uid;
  memcpy(&uid, id, 128);
  ncclComm_t comm = nullptr;
  if (!nccl_ok(a.comm_init_rank(&comm, world, uid, rank), "ncclCommInitRank", err)) return false;
  c.comm = comm;
  c.rank = rank;
  c.world = world;
  return true;
}

void ep_comm_destroy(EpComm& c) {
  if (c.comm && nccl().ok) nccl().comm_destroy((ncclComm_t)c.comm);
  c.comm = nullptr;
}

bool ep_allgather_i32(const EpComm& c, const int32_t* send, int32_t* recv, int count, cudaStream_t s,
                      std::string& err) {
  return nccl_ok(nccl().all_gather(send, recv, (size_t)count, ncclInt32, (ncclComm_t)c.comm, s), "ncclAllGather",
                 err);
}

bool ep_exchange(const EpComm& c, const float* send, const int32_t* send_tag, const int* send_counts,
                 const int* send_off, float* recv, int32_t* recv_tag, const int* recv_counts, const int* recv_off,
                 int width, cudaStream_t s, std::string& err) {
  const NcclApi& a = nccl();
  ncclComm_t comm = (ncclComm_t)c.comm;
  if (!nccl_ok(a.group_start(), "ncclGroupStart", err)) return false;
  bool ok = true;
  for (int p = 0; p < c.world && ok; p++) {
    if (send_counts[p]) {
      ok = nccl_ok(a.send(send + (size_t)send_off[p] * width, (size_t)send_counts[p] * width, ncclFloat32, p, comm, s),
                   "ncclSend", err);
      if (ok && send_tag)
        ok = nccl_ok(a.send(send_tag + send_off[p], (size_t)send_counts[p], ncclInt32, p, comm, s), "ncclSend", err);
    }
    if (ok && recv_counts[p]) {
      ok = nccl_ok(a.recv(recv + (size_t)recv_off[p] * width, (size_t)recv_counts[p] * width, ncclFloat32, p, comm, s),
                   "ncclRecv", err);
      if (ok && recv_tag)
        ok = nccl_ok(a.recv(recv_tag + recv_off[p], (size_t)recv_counts[p], ncclInt32, p, comm, s), "ncclRecv", err);
    }
  }
  // the group is closed on every path so that NCCL's state stays consistent
  std::string e2;
  const bool closed = nccl_ok(a.group_end(), "ncclGroupEnd", e2);
  if (ok && !closed) err = e2;
  return ok && closed;
}

void ep_pack(const float* rows, const int32_t* sel, const int32_t* order, int n, float* send, int32_t* tag,
             cudaStream_t s) {
  if (n > 0) k_ep_pack<<<n, 128, 0, s>>>(rows, sel, order, n, send, tag);
}

void ep_fake_sel(const int32_t* tag, int n, int pad, int32_t* sel4, cudaStream_t s) {
  const int n4 = (n + N_USED - 1) / N_USED * N_USED;
  if (n4 > 0) k_ep_fake_sel<<<(n4 + 255) / 256, 256, 0, s>>>(tag, n, pad, sel4);
}

void ep_unpack(const float* back, const int32_t* order, int n, float* out, cudaStream_t s) {
  if (n > 0) k_ep_unpack<<<n, 128, 0, s>>>(back, order, n, out);
}

}  // namespace lfm
