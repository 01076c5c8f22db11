// ep_link.h — the token exchange of an expert-parallel engine: an all-to-all
// of variable byte counts between the ranks of one group, issued on the
// engine's stream. Two implementations:
//   * NCCL: grouped ncclSend/ncclRecv (one process per GPU, over NVLink). The
//     library is opened at run time (dlopen "libnccl.so.2"), so a process that
//     already loaded NCCL (PyTorch does) shares that copy.
//   * hub: engines of one process exchange through a shared object (device
//     copies between their buffers, host barriers) - several ranks on one GPU
//     for tests; no kernel waits on another.
// Every wait is bounded: a rank that never arrives makes the others return
// CHALOT_ERR_TIMEOUT instead of hanging.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>

namespace chalot {

class EpLink {
 public:
  virtual ~EpLink() = default;
  int rank() const { return rank_; }
  int world() const { return world_; }
  // Rank r sends send_bytes[g] bytes starting at send + sum(send_bytes[0..g))
  // to rank g, and receives recv_bytes[g] bytes from rank g at recv +
  // sum(recv_bytes[0..g)). The sizes must agree pairwise across the ranks.
  // Returns a CHALOT_ status; *msg explains a failure.
  virtual int all_to_all(const void* send, const size_t* send_bytes, void* recv, const size_t* recv_bytes,
                         cudaStream_t s, std::string* msg) = 0;
  // Waits for the stream, bounded (a peer that died shows up here).
  virtual int sync(cudaStream_t s, std::string* msg) = 0;

 protected:
  int rank_ = 0, world_ = 1;
};

// NCCL: `id` is the 128-byte ncclUniqueId rank 0 created (ep_nccl_unique_id)
// and every rank received out of band.
int ep_nccl_unique_id(uint8_t id[128], std::string* msg);
int ep_nccl_link(int rank, int world, const uint8_t id[128], int device, std::unique_ptr<EpLink>* out,
                 std::string* msg);

// Hub: one shared object per group of in-process ranks.
struct EpHub;
EpHub* ep_hub_create(int world);
int ep_hub_world(const EpHub* hub);
void ep_hub_release(EpHub* hub);  // drops one reference (creator + every link)
int ep_hub_link(EpHub* hub, int rank, std::unique_ptr<EpLink>* out, std::string* msg);

// Bound of every wait on a peer.
constexpr double kEpTimeoutSeconds = 120.0;

}  // namespace chalot
