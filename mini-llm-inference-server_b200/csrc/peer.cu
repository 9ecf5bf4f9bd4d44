// Shared device memory between the processes of one node (CUDA IPC) and a flag barrier over it: the
// transport of the output all-gather that KV-head sharding needs.
//
// The attention kernel leaves this rank's unsplit rows in its own gathered buffer; the split-K reduction
// (mlb_splitk_reduce_gather) finishes the split rows and stores every row of this rank into every peer's
// buffer (mlb_out_targets, addresses from mlb_ipc_open, reached over NVLink).  What is left is to know
// that every peer's rows have landed: peer_barrier_kernel, launched after them on the stream, fences at
// system scope, raises this rank's word in every peer's flag array to the next epoch with a release
// store, and waits (acquire loads, bounded in time and in iterations) until every peer has raised its word
// in this rank's array.  The epoch lives in device memory and the kernel advances it, so a CUDA graph that
// captured the barrier stays in step when it is replayed.
#include <cstring>
#include <string>

#include "attn_args.cuh"
#include "peer.cuh"

namespace mlb {
int set_last_error(int code, const char* msg);  // the mlb_last_error() channel (capi.cu)
}  // namespace mlb

namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == MLB_IPC_HANDLE_BYTES, "IPC handle size");

// One warp: the whole barrier (the stream's earlier writes are ordered before the flags by the fence in
// peer_signal_and_wait).
__global__ void __launch_bounds__(32) peer_barrier_kernel(const mlb::PeerSync ps, int32_t* err) {
  mlb::griddep_begin();
  if (mlb::peer_signal_and_wait(ps, threadIdx.x) && threadIdx.x == 0) mlb::flag_error(err, MLB_DEV_WAIT_TIMEOUT);
}

int peer_fail(int code, const std::string& msg) { return mlb::set_last_error(code, msg.c_str()); }

int peer_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MLB_OK;
  return peer_fail(MLB_ECUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

}  // namespace

extern "C" {

int mlb_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle) {
  if (bytes <= 0 || !dev_ptr || !handle) return peer_fail(MLB_EINVAL, "ipc_alloc: bad arguments");
  void* p = nullptr;
  if (int rc = peer_cuda(cudaMalloc(&p, static_cast<size_t>(bytes)), "ipc_alloc: cudaMalloc")) return rc;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  // the zeros must be in place before any peer can open the handle and raise a flag in it
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return peer_cuda(e, "ipc_alloc");
  }
  std::memcpy(handle, &h, sizeof h);
  *dev_ptr = p;
  return MLB_OK;
}

int mlb_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return peer_fail(MLB_EINVAL, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void* p = nullptr;
  if (int rc = peer_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "ipc_open")) return rc;
  *dev_ptr = p;
  return MLB_OK;
}

int mlb_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return MLB_OK;
  return peer_cuda(cudaIpcCloseMemHandle(dev_ptr), "ipc_close");
}

int mlb_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return MLB_OK;
  return peer_cuda(cudaFree(dev_ptr), "ipc_free");
}

int mlb_peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t* epoch, int64_t timeout_ns,
                     int32_t* err_word, void* stream) {
  if (world < 1 || world > MLB_MAX_OUT_DESTS || rank < 0 || rank >= world)
    return peer_fail(MLB_EINVAL, "peer_barrier: rank " + std::to_string(rank) + " of " + std::to_string(world) +
                                     " (1.." + std::to_string(MLB_MAX_OUT_DESTS) + " ranks)");
  if (!flags || !epoch) return peer_fail(MLB_EINVAL, "peer_barrier: null pointer");
  if (timeout_ns < 0) return peer_fail(MLB_EINVAL, "peer_barrier: negative timeout");
  mlb::PeerSync ps{};
  for (int i = 0; i < world; ++i) {
    if (!flags[i]) return peer_fail(MLB_EINVAL, "peer_barrier: flag array " + std::to_string(i) + " is null");
    ps.flags[i] = flags[i];
  }
  ps.epoch = epoch;
  ps.rank = rank;
  ps.world = world;
  ps.timeout_ns = timeout_ns;
  return peer_cuda(mlb::launch_k(peer_barrier_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), ps,
                                 err_word),
                   "peer_barrier launch");
}

}  // extern "C"
