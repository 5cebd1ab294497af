// comm.cu -- the one collective of a multi-GPU job: the final gather of generated token ids.
//
// Sequences are independent (ane/stories/infer.go:136-245 decodes one sequence with no shared
// state), so a job of n_total sequences is split across ranks (one process per GPU) in
// contiguous blocks: rank r owns [r*base + min(r, extra), ...) with base, extra = divmod(n_total,
// nranks), the first `extra` ranks holding one more.  Nothing crosses ranks while tokens are
// generated; at the end llm_gather_tokens brings every rank's [steps][n_local] block of token ids
// to every rank in global sequence order with one NCCL all-gather over NVLink / NVSwitch.
//
// NCCL is loaded when the first communicator is created (dlopen of libnccl.so.2; a process that
// already loaded NCCL, e.g. through torch.distributed, shares that copy), so the library itself
// does not depend on NCCL.  Communicators are created non-blocking and every wait is bounded
// on the host: a rank that never joins makes the others' call fail with LLM_ERR_DEVICE after
// the timeout (the communicator is aborted) instead of waiting forever.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/llm_cuda.h"

int llm_detail_fail(int code, const char* msg);

namespace {

int fail_fmt(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  return llm_detail_fail(code, buf);
}

struct Nccl {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
};

std::mutex g_nccl_mu;
Nccl g_nccl;

int load_nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.ok) return LLM_OK;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
  if (!h) return fail_fmt(LLM_ERR_UNSUPPORTED, "NCCL is not available: %s", dlerror());
  auto sym = [&](const char* n) { return dlsym(h, n); };
  g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(sym("ncclGetUniqueId"));
  g_nccl.init_rank_config = reinterpret_cast<decltype(g_nccl.init_rank_config)>(sym("ncclCommInitRankConfig"));
  g_nccl.async_error = reinterpret_cast<decltype(g_nccl.async_error)>(sym("ncclCommGetAsyncError"));
  g_nccl.abort = reinterpret_cast<decltype(g_nccl.abort)>(sym("ncclCommAbort"));
  g_nccl.destroy = reinterpret_cast<decltype(g_nccl.destroy)>(sym("ncclCommDestroy"));
  g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(sym("ncclAllGather"));
  g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(sym("ncclGetErrorString"));
  if (!g_nccl.get_unique_id || !g_nccl.init_rank_config || !g_nccl.async_error || !g_nccl.abort || !g_nccl.destroy ||
      !g_nccl.all_gather || !g_nccl.error_string)
    return fail_fmt(LLM_ERR_UNSUPPORTED, "NCCL library lacks a required symbol");
  g_nccl.ok = true;
  return LLM_OK;
}

}  // namespace

struct llm_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0, device = 0;
  double timeout_s = 60.0;
  cudaStream_t stream = nullptr;
  int32_t *d_send = nullptr, *d_recv = nullptr;
  size_t cap = 0;  // int32 elements of d_send
  cudaEvent_t e0 = nullptr, e1 = nullptr;  // around the last gather's copy-in and all-gather
  bool timed = false;
};

namespace {

using Clock = std::chrono::steady_clock;

// Poll the communicator until its pending operation (init) finished; bounded.
int wait_comm(llm_comm* c, const char* what) {
  const auto t0 = Clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = g_nccl.async_error(c->comm, &st);
    if (r != ncclSuccess) return fail_fmt(LLM_ERR_DEVICE, "%s: %s", what, g_nccl.error_string(r));
    if (st == ncclSuccess) return LLM_OK;
    if (st != ncclInProgress) return fail_fmt(LLM_ERR_DEVICE, "%s: %s", what, g_nccl.error_string(st));
    if (std::chrono::duration<double>(Clock::now() - t0).count() > c->timeout_s) {
      g_nccl.abort(c->comm);
      c->comm = nullptr;
      return fail_fmt(LLM_ERR_DEVICE, "%s: timed out after %.0f s (a rank did not join)", what, c->timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

// Wait for the collective on c->stream; bounded.  A non-blocking communicator may still be
// enqueueing the collective when the call returns (ncclInProgress): the stream is only polled
// once the communicator reports the enqueue done, else an idle stream would look finished.
int wait_stream(llm_comm* c, const char* what) {
  const auto t0 = Clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = g_nccl.async_error(c->comm, &st);
    if (r != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
      const ncclResult_t bad = r != ncclSuccess ? r : st;
      g_nccl.abort(c->comm);
      c->comm = nullptr;
      return fail_fmt(LLM_ERR_DEVICE, "%s: %s", what, g_nccl.error_string(bad));
    }
    if (st == ncclSuccess) {
      const cudaError_t e = cudaStreamQuery(c->stream);
      if (e == cudaSuccess) return LLM_OK;
      if (e != cudaErrorNotReady) return fail_fmt(LLM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    }
    if (std::chrono::duration<double>(Clock::now() - t0).count() > c->timeout_s) {
      g_nccl.abort(c->comm);  // ends the collective's kernels; the communicator is unusable
      c->comm = nullptr;
      return fail_fmt(LLM_ERR_DEVICE, "%s: timed out after %.0f s (a rank did not take part)", what, c->timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace

extern "C" int llm_shard_range(int n_total, int nranks, int rank, int* start, int* count) {
  if (!start || !count) return fail_fmt(LLM_ERR_INVALID, "nil output");
  if (nranks <= 0 || rank < 0 || rank >= nranks) return fail_fmt(LLM_ERR_INVALID, "rank %d out of range for %d ranks", rank, nranks);
  if (n_total < 0) return fail_fmt(LLM_ERR_INVALID, "sequence count %d is negative", n_total);
  const int base = n_total / nranks, extra = n_total % nranks;
  *start = rank * base + (rank < extra ? rank : extra);
  *count = base + (rank < extra ? 1 : 0);
  return LLM_OK;
}

extern "C" int llm_comm_unique_id(unsigned char* id, size_t id_bytes) {
  if (!id || id_bytes < sizeof(ncclUniqueId)) return fail_fmt(LLM_ERR_INVALID, "id buffer needs %zu bytes", sizeof(ncclUniqueId));
  int rc = load_nccl();
  if (rc) return rc;
  ncclUniqueId u;
  const ncclResult_t r = g_nccl.get_unique_id(&u);
  if (r != ncclSuccess) return fail_fmt(LLM_ERR_DEVICE, "ncclGetUniqueId: %s", g_nccl.error_string(r));
  memcpy(id, &u, sizeof u);
  return LLM_OK;
}

extern "C" int llm_comm_create(const unsigned char* id, size_t id_bytes, int nranks, int rank, int device,
                               double timeout_s, llm_comm** out) {
  if (!id || !out || id_bytes < sizeof(ncclUniqueId)) return fail_fmt(LLM_ERR_INVALID, "bad arguments");
  if (nranks <= 0 || rank < 0 || rank >= nranks) return fail_fmt(LLM_ERR_INVALID, "rank %d out of range for %d ranks", rank, nranks);
  int rc = load_nccl();
  if (rc) return rc;
  if (cudaSetDevice(device) != cudaSuccess) return fail_fmt(LLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  auto* c = new llm_comm();
  c->nranks = nranks;
  c->rank = rank;
  c->device = device;
  c->timeout_s = timeout_s > 0 ? timeout_s : 60.0;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&c->e0) != cudaSuccess || cudaEventCreate(&c->e1) != cudaSuccess) {
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return fail_fmt(LLM_ERR_CUDA, "stream creation failed");
  }
  ncclUniqueId u;
  memcpy(&u, id, sizeof u);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const ncclResult_t r = g_nccl.init_rank_config(&c->comm, nranks, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    cudaStreamDestroy(c->stream);
    delete c;
    return fail_fmt(LLM_ERR_DEVICE, "ncclCommInitRankConfig: %s", g_nccl.error_string(r));
  }
  rc = wait_comm(c, "communicator init");
  if (rc) {
    if (c->comm) g_nccl.abort(c->comm);
    cudaStreamDestroy(c->stream);
    delete c;
    return rc;
  }
  *out = c;
  return LLM_OK;
}

extern "C" int llm_comm_destroy(llm_comm* c) {
  if (!c) return LLM_OK;
  cudaSetDevice(c->device);
  if (c->comm) g_nccl.destroy(c->comm);
  if (c->d_send) cudaFree(c->d_send);
  if (c->d_recv) cudaFree(c->d_recv);
  if (c->e0) cudaEventDestroy(c->e0);
  if (c->e1) cudaEventDestroy(c->e1);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return LLM_OK;
}

extern "C" int llm_comm_last_gather_ms(llm_comm* c, double* ms) {
  if (!c || !ms) return fail_fmt(LLM_ERR_INVALID, "nil argument");
  if (!c->timed) return fail_fmt(LLM_ERR_STATE, "no gather has completed");
  float v = 0.f;
  if (cudaEventElapsedTime(&v, c->e0, c->e1) != cudaSuccess) return fail_fmt(LLM_ERR_CUDA, "event timing failed");
  *ms = v;
  return LLM_OK;
}

extern "C" int llm_gather_tokens(llm_comm* c, const int32_t* tokens, int steps, int n_local, int n_total, int32_t* out) {
  if (!c || !tokens || !out) return fail_fmt(LLM_ERR_INVALID, "nil argument");
  if (!c->comm) return fail_fmt(LLM_ERR_STATE, "communicator was aborted");
  if (steps < 0) return fail_fmt(LLM_ERR_INVALID, "steps %d is negative", steps);
  int start = 0, count = 0;
  int rc = llm_shard_range(n_total, c->nranks, c->rank, &start, &count);
  if (rc) return rc;
  if (n_local != count)
    return fail_fmt(LLM_ERR_INVALID, "rank %d holds %d sequences, its shard has %d", c->rank, n_local, count);
  int width = 0, s0 = 0;
  llm_shard_range(n_total, c->nranks, 0, &s0, &width);  // the largest shard
  const size_t per = static_cast<size_t>(steps) * width;
  if (per == 0) return LLM_OK;
  if (cudaSetDevice(c->device) != cudaSuccess) return fail_fmt(LLM_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
  if (per > c->cap) {
    if (c->d_send) cudaFree(c->d_send);
    if (c->d_recv) cudaFree(c->d_recv);
    c->d_send = c->d_recv = nullptr;
    if (cudaMalloc(&c->d_send, per * 4) != cudaSuccess ||
        cudaMalloc(&c->d_recv, per * 4 * static_cast<size_t>(c->nranks)) != cudaSuccess) {
      c->cap = 0;
      return fail_fmt(LLM_ERR_OOM, "gather buffers of %zu bytes", per * 4 * (1 + static_cast<size_t>(c->nranks)));
    }
    c->cap = per;
  }
  // this rank's block padded to the largest shard with -1
  std::vector<int32_t> send(per, -1);
  for (int s = 0; s < steps; ++s) memcpy(send.data() + static_cast<size_t>(s) * width, tokens + static_cast<size_t>(s) * n_local, n_local * 4);
  c->timed = false;
  cudaEventRecord(c->e0, c->stream);
  if (cudaMemcpyAsync(c->d_send, send.data(), per * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
    return fail_fmt(LLM_ERR_CUDA, "copy of the token block failed");
  const ncclResult_t r = g_nccl.all_gather(c->d_send, c->d_recv, per, ncclInt32, c->comm, c->stream);
  if (r != ncclSuccess && r != ncclInProgress) return fail_fmt(LLM_ERR_DEVICE, "ncclAllGather: %s", g_nccl.error_string(r));
  rc = wait_stream(c, "token gather");
  if (rc) return rc;
  cudaEventRecord(c->e1, c->stream);
  cudaEventSynchronize(c->e1);
  c->timed = true;
  std::vector<int32_t> recv(per * c->nranks);
  if (cudaMemcpy(recv.data(), c->d_recv, per * 4 * c->nranks, cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail_fmt(LLM_ERR_CUDA, "copy of the gathered tokens failed");
  for (int r2 = 0; r2 < c->nranks; ++r2) {
    int st = 0, cnt = 0;
    llm_shard_range(n_total, c->nranks, r2, &st, &cnt);
    const int32_t* blk = recv.data() + per * r2;
    for (int s = 0; s < steps; ++s)
      memcpy(out + static_cast<size_t>(s) * n_total + st, blk + static_cast<size_t>(s) * width, cnt * 4);
  }
  return LLM_OK;
}
