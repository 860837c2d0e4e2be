// Data-parallel communicator over NCCL (NVLink / NVSwitch inside one box).
// The reference is single-device (src/device.rs:37-41); this is the one
// exchange the data-parallel training step adds: a mean all-reduce of the
// gradients.  Init is non-blocking and polled against a host deadline so a
// rank that never joins turns into an error instead of a hang.
//
// NCCL is resolved with dlopen at first use instead of being linked: a
// process that also loads torch must share torch's libnccl.so.2 (same
// SONAME, already resident), and linking the system copy would make it win.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "fg_comm.h"
#include "fg_internal.h"

struct fg_comm {
  ncclComm_t comm;
  int rank;
  int nranks;
  int timeout_ms;
};

namespace fg {

struct Nccl {
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRankConfig) commInitRankConfig = nullptr;
  decltype(&ncclCommGetAsyncError) commGetAsyncError = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
  decltype(&ncclCommFinalize) commFinalize = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclCommAbort) commAbort = nullptr;
  decltype(&ncclGetErrorString) getErrorString = nullptr;
  bool ok = false;
  std::string why;
};

static Nccl *nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      n.why = dlerror();
      return;
    }
#define FG_SYM(field, name)                                 \
  n.field = (decltype(n.field))dlsym(h, name);              \
  if (!n.field) {                                           \
    n.why = std::string("missing NCCL symbol ") + name;     \
    return;                                                 \
  }
    FG_SYM(getUniqueId, "ncclGetUniqueId")
    FG_SYM(commInitRankConfig, "ncclCommInitRankConfig")
    FG_SYM(commGetAsyncError, "ncclCommGetAsyncError")
    FG_SYM(allReduce, "ncclAllReduce")
    FG_SYM(commFinalize, "ncclCommFinalize")
    FG_SYM(commDestroy, "ncclCommDestroy")
    FG_SYM(commAbort, "ncclCommAbort")
    FG_SYM(getErrorString, "ncclGetErrorString")
#undef FG_SYM
    n.ok = true;
  });
  return &n;
}

#define FG_NCCL_REQUIRE()                                                              \
  do {                                                                                 \
    if (!fg::nccl()->ok)                                                               \
      return fg::set_error(FG_ERR_NCCL, "NCCL unavailable: %s", fg::nccl()->why.c_str()); \
  } while (0)

// Wait until the communicator's last operation left ncclInProgress.
static int nccl_settle(fg_comm *c, ncclResult_t r, const char *what) {
  auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    ncclResult_t ar = ncclSuccess;
    nccl()->commGetAsyncError(c->comm, &ar);
    r = ar;
    if (r != ncclInProgress) break;
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0)
                  .count();
    if (ms > c->timeout_ms) {
      return set_error(FG_ERR_NCCL, "%s: timed out after %d ms", what, c->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  if (r != ncclSuccess)
    return set_error(FG_ERR_NCCL, "%s failed: %s", what, nccl()->getErrorString(r));
  return FG_OK;
}

int comm_allreduce_mean(fg_comm *c, float *buf, size_t count, cudaStream_t st) {
  if (!count) return FG_OK;
  ncclResult_t r = nccl()->allReduce(buf, buf, count, ncclFloat32, ncclAvg, c->comm, st);
  return nccl_settle(c, r, "ncclAllReduce");
}

// Plain sum (callers pre-scale by 1/nranks): unlike ncclAvg it is eligible
// for NVLS, the in-switch reduction over NVSwitch multicast.
int comm_allreduce_sum(fg_comm *c, float *buf, size_t count, cudaStream_t st) {
  if (!count) return FG_OK;
  ncclResult_t r = nccl()->allReduce(buf, buf, count, ncclFloat32, ncclSum, c->comm, st);
  return nccl_settle(c, r, "ncclAllReduce");
}

int comm_nranks(const fg_comm *c) { return c ? c->nranks : 1; }

// The backward GEMMs of config 5 have 128 x (a power of two) output tiles
// at every rank count, so a persistent grid of num_SMs - 20 = 128 CTAs on a
// B200 loses nothing to tile quantisation, and the 20 SMs it leaves free
// run the all-reduce beside it.  The collective must then fit in those SMs:
// a wider one would take SMs the GEMM's 128 CTAs need and push some of its
// tiles into a second wave.
int comm_sm_reserve() {
  const char *e = getenv("FG_COMM_SM_RESERVE");
  int v = e && *e ? atoi(e) : kCommSmReserve;
  return v < 0 ? 0 : (v > 64 ? 64 : v);
}

}  // namespace fg

extern "C" {

int fg_comm_unique_id(char out[FG_UNIQUE_ID_BYTES]) {
  FG_REQUIRE(out, "fg_comm_unique_id: null output");
  static_assert(sizeof(ncclUniqueId) == FG_UNIQUE_ID_BYTES, "NCCL unique id size");
  FG_NCCL_REQUIRE();
  ncclUniqueId id;
  ncclResult_t r = fg::nccl()->getUniqueId(&id);
  if (r != ncclSuccess)
    return fg::set_error(FG_ERR_NCCL, "ncclGetUniqueId: %s", fg::nccl()->getErrorString(r));
  memcpy(out, &id, sizeof(id));
  return FG_OK;
}

int fg_comm_init(int rank, int nranks, const char uid[FG_UNIQUE_ID_BYTES], int timeout_ms,
                 fg_comm **out) {
  FG_REQUIRE(out && uid, "fg_comm_init: null argument");
  FG_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "fg_comm_init: bad rank %d of %d", rank,
             nranks);
  FG_NCCL_REQUIRE();
  ncclUniqueId id;
  memcpy(&id, uid, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  if (fg::comm_sm_reserve() > 0) cfg.maxCTAs = fg::comm_sm_reserve();
  fg_comm *c = new fg_comm{nullptr, rank, nranks, timeout_ms > 0 ? timeout_ms : 60000};
  ncclResult_t r = fg::nccl()->commInitRankConfig(&c->comm, nranks, id, rank, &cfg);
  int rc = (r == ncclSuccess || r == ncclInProgress) && c->comm
               ? fg::nccl_settle(c, r, "ncclCommInitRankConfig")
               : fg::set_error(FG_ERR_NCCL, "ncclCommInitRankConfig: %s", fg::nccl()->getErrorString(r));
  if (rc != FG_OK) {
    if (c->comm) fg::nccl()->commAbort(c->comm);
    delete c;
    return rc;
  }
  *out = c;
  return FG_OK;
}

int fg_comm_destroy(fg_comm *comm) {
  if (!comm) return FG_OK;
  ncclResult_t r = fg::nccl()->commFinalize(comm->comm);
  int rc = fg::nccl_settle(comm, r, "ncclCommFinalize");
  fg::nccl()->commDestroy(comm->comm);
  delete comm;
  return rc;
}

int fg_comm_abort(fg_comm *comm) {
  if (!comm) return FG_OK;
  fg::nccl()->commAbort(comm->comm);
  delete comm;
  return FG_OK;
}

int fg_allreduce_mean_f32(fg_comm *comm, float *d_buf, size_t count, void *stream) {
  FG_REQUIRE(comm && (count == 0 || d_buf), "fg_allreduce_mean_f32: null argument");
  return fg::comm_allreduce_mean(comm, d_buf, count, (cudaStream_t)stream);
}

}  // extern "C"
