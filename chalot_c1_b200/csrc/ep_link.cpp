// ep_link.cpp — NCCL and in-process implementations of the expert-parallel
// token exchange (ep_link.h).
#include "ep_link.h"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <thread>
#include <type_traits>
#include <vector>

#include "capi_internal.h"

namespace chalot {
namespace {

using Clock = std::chrono::steady_clock;

double seconds_since(Clock::time_point t0) {
  return std::chrono::duration<double>(Clock::now() - t0).count();
}

// ---- NCCL, opened at run time ---------------------------------------------

struct NcclApi {
  bool ok = false;
  std::string why;
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.why = std::string("cannot open libnccl.so.2: ") + dlerror();
      return a;
    }
    auto get = [&](const char* name, auto* fn) {
      *fn = reinterpret_cast<std::remove_reference_t<decltype(*fn)>>(dlsym(h, name));
      if (!*fn && a.why.empty()) a.why = std::string("libnccl lacks ") + name;
    };
    get("ncclGetUniqueId", &a.get_unique_id);
    get("ncclCommInitRank", &a.init_rank);
    get("ncclCommDestroy", &a.destroy);
    get("ncclCommAbort", &a.abort);
    get("ncclCommGetAsyncError", &a.async_error);
    get("ncclSend", &a.send);
    get("ncclRecv", &a.recv);
    get("ncclGroupStart", &a.group_start);
    get("ncclGroupEnd", &a.group_end);
    get("ncclGetErrorString", &a.error_string);
    a.ok = a.why.empty();
    return a;
  }();
  return api;
}

class NcclLink final : public EpLink {
 public:
  NcclLink(int rank, int world, ncclComm_t comm) : comm_(comm) {
    rank_ = rank;
    world_ = world;
  }
  ~NcclLink() override {
    if (comm_) {
      if (failed_)
        nccl().abort(comm_);
      else
        nccl().destroy(comm_);
    }
  }

  int all_to_all(const void* send, const size_t* send_bytes, void* recv, const size_t* recv_bytes, cudaStream_t s,
                 std::string* msg) override {
    if (failed_) {
      *msg = "NCCL link failed earlier";
      return CHALOT_ERR_NCCL;
    }
    const NcclApi& n = nccl();
    const char* sp = static_cast<const char*>(send);
    char* rp = static_cast<char*>(recv);
    ncclResult_t r = n.group_start();
    size_t so = 0, ro = 0;
    for (int g = 0; g < world_ && r == ncclSuccess; ++g) {
      if (send_bytes[g]) r = n.send(sp + so, send_bytes[g], ncclInt8, g, comm_, s);
      if (r == ncclSuccess && recv_bytes[g]) r = n.recv(rp + ro, recv_bytes[g], ncclInt8, g, comm_, s);
      so += send_bytes[g];
      ro += recv_bytes[g];
    }
    const ncclResult_t e = n.group_end();
    if (r == ncclSuccess) r = e;
    if (r != ncclSuccess) {
      failed_ = true;
      *msg = std::string("NCCL all-to-all: ") + n.error_string(r);
      return CHALOT_ERR_NCCL;
    }
    return CHALOT_OK;
  }

  int sync(cudaStream_t s, std::string* msg) override {
    const auto t0 = Clock::now();
    for (;;) {
      const cudaError_t q = cudaStreamQuery(s);
      if (q == cudaSuccess) return CHALOT_OK;
      if (q != cudaErrorNotReady) {
        *msg = std::string("EP sync: ") + cudaGetErrorString(q);
        return CHALOT_ERR_CUDA;
      }
      ncclResult_t ae = ncclSuccess;
      nccl().async_error(comm_, &ae);
      if (ae != ncclSuccess && ae != ncclInProgress) {
        failed_ = true;
        *msg = std::string("NCCL: ") + nccl().error_string(ae);
        return CHALOT_ERR_NCCL;
      }
      if (seconds_since(t0) > kEpTimeoutSeconds) {
        failed_ = true;
        *msg = "EP sync: a peer did not answer within the time limit";
        return CHALOT_ERR_TIMEOUT;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }

 private:
  ncclComm_t comm_ = nullptr;
  bool failed_ = false;
};

}  // namespace

int ep_nccl_unique_id(uint8_t id[128], std::string* msg) {
  const NcclApi& n = nccl();
  if (!n.ok) {
    *msg = n.why;
    return CHALOT_ERR_NCCL;
  }
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId u;
  const ncclResult_t r = n.get_unique_id(&u);
  if (r != ncclSuccess) {
    *msg = std::string("ncclGetUniqueId: ") + n.error_string(r);
    return CHALOT_ERR_NCCL;
  }
  std::memcpy(id, &u, 128);
  return CHALOT_OK;
}

int ep_nccl_link(int rank, int world, const uint8_t id[128], int device, std::unique_ptr<EpLink>* out,
                 std::string* msg) {
  const NcclApi& n = nccl();
  if (!n.ok) {
    *msg = n.why;
    return CHALOT_ERR_NCCL;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    *msg = "cudaSetDevice failed";
    return CHALOT_ERR_CUDA;
  }
  ncclUniqueId u;
  std::memcpy(&u, id, 128);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = n.init_rank(&comm, world, u, rank);
  if (r != ncclSuccess) {
    *msg = std::string("ncclCommInitRank: ") + n.error_string(r);
    return CHALOT_ERR_NCCL;
  }
  out->reset(new NcclLink(rank, world, comm));
  return CHALOT_OK;
}

// ---- in-process hub -------------------------------------------------------

struct EpHub {
  explicit EpHub(int w) : world(w), posts(w), refs(1) {}
  struct Post {
    const char* send = nullptr;
    std::vector<size_t> bytes;  // per destination
    cudaEvent_t ready = nullptr;
  };
  const int world;
  std::mutex m;
  std::condition_variable cv;
  std::vector<Post> posts;
  uint64_t round = 0;
  int arrived = 0, done = 0;
  int refs;
  bool broken = false;
};

namespace {

class HubLink final : public EpLink {
 public:
  HubLink(EpHub* hub, int rank) : hub_(hub) {
    rank_ = rank;
    world_ = hub->world;
    cudaEventCreateWithFlags(&ready_, cudaEventDisableTiming);
  }
  ~HubLink() override {
    if (ready_) cudaEventDestroy(ready_);
    ep_hub_release(hub_);
  }

  int all_to_all(const void* send, const size_t* send_bytes, void* recv, const size_t* recv_bytes, cudaStream_t s,
                 std::string* msg) override {
    EpHub& h = *hub_;
    if (cudaEventRecord(ready_, s) != cudaSuccess) {
      *msg = "hub: event record failed";
      return CHALOT_ERR_CUDA;
    }
    std::unique_lock<std::mutex> lk(h.m);
    if (h.broken) {
      *msg = "hub: the group failed earlier";
      return CHALOT_ERR_STATE;
    }
    const uint64_t r = h.round;
    h.posts[rank_].send = static_cast<const char*>(send);
    h.posts[rank_].bytes.assign(send_bytes, send_bytes + world_);
    h.posts[rank_].ready = ready_;
    if (++h.arrived == world_) h.cv.notify_all();
    if (!wait(lk, [&] { return h.arrived == world_ || h.round != r || h.broken; }, msg)) return CHALOT_ERR_TIMEOUT;
    // every rank posted: pull my parts from each source's send buffer
    char* rp = static_cast<char*>(recv);
    size_t ro = 0;
    int rc = CHALOT_OK;
    for (int g = 0; g < world_ && rc == CHALOT_OK; ++g) {
      const EpHub::Post& p = h.posts[g];
      size_t off = 0;
      for (int k = 0; k < rank_; ++k) off += p.bytes[k];
      if (p.bytes[rank_] != recv_bytes[g]) {
        *msg = "hub: send and receive sizes disagree";
        rc = CHALOT_ERR_ARG;
        break;
      }
      if (cudaStreamWaitEvent(s, p.ready, 0) != cudaSuccess ||
          (recv_bytes[g] &&
           cudaMemcpyAsync(rp + ro, p.send + off, recv_bytes[g], cudaMemcpyDeviceToDevice, s) != cudaSuccess)) {
        *msg = "hub: device copy failed";
        rc = CHALOT_ERR_CUDA;
      }
      ro += recv_bytes[g];
    }
    // the sources' buffers must outlive the copies: finish them, then wait for all
    lk.unlock();
    if (rc == CHALOT_OK && cudaStreamSynchronize(s) != cudaSuccess) {
      *msg = "hub: stream failed";
      rc = CHALOT_ERR_CUDA;
    }
    lk.lock();
    if (rc != CHALOT_OK) {
      h.broken = true;
      h.cv.notify_all();
      return rc;
    }
    if (++h.done == world_) {
      h.done = 0;
      h.arrived = 0;
      ++h.round;
      h.cv.notify_all();
      return CHALOT_OK;
    }
    if (!wait(lk, [&] { return h.round != r || h.broken; }, msg)) return CHALOT_ERR_TIMEOUT;
    if (h.broken) {
      *msg = "hub: a peer failed";
      return CHALOT_ERR_STATE;
    }
    return CHALOT_OK;
  }

  int sync(cudaStream_t s, std::string* msg) override {
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) return CHALOT_OK;
    *msg = std::string("EP sync: ") + cudaGetErrorString(e);
    return CHALOT_ERR_CUDA;
  }

 private:
  template <class P>
  bool wait(std::unique_lock<std::mutex>& lk, P pred, std::string* msg) {
    const auto limit = std::chrono::duration<double>(kEpTimeoutSeconds);
    if (hub_->cv.wait_for(lk, limit, pred)) return true;
    hub_->broken = true;
    hub_->cv.notify_all();
    *msg = "hub: a peer did not arrive within the time limit";
    return false;
  }

  EpHub* hub_;
  cudaEvent_t ready_ = nullptr;
};

}  // namespace

EpHub* ep_hub_create(int world) { return new EpHub(world); }

int ep_hub_world(const EpHub* hub) { return hub ? hub->world : 0; }

void ep_hub_release(EpHub* hub) {
  if (!hub) return;
  bool last;
  {
    std::lock_guard<std::mutex> g(hub->m);
    last = --hub->refs == 0;
  }
  if (last) delete hub;
}

int ep_hub_link(EpHub* hub, int rank, std::unique_ptr<EpLink>* out, std::string* msg) {
  if (!hub || rank < 0 || rank >= hub->world) {
    *msg = "hub: bad rank";
    return CHALOT_ERR_ARG;
  }
  {
    std::lock_guard<std::mutex> g(hub->m);
    ++hub->refs;
  }
  out->reset(new HubLink(hub, rank));
  return CHALOT_OK;
}

}  // namespace chalot
