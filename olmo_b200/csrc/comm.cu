// Stand-alone launches of the peer-memory collectives (comm.cuh), the flag signal and the small scalar all-reduce
// that doubles as the end-of-step barrier.
#include "comm.cuh"
#include "api.h"

namespace ob {
namespace {

constexpr int COMM_THREADS = 512;

__global__ void __launch_bounds__(COMM_THREADS) comm_kernel(const __grid_constant__ CommTask task) {
  __shared__ CommScratch scratch;
  const CommGroup g = {static_cast<int>(threadIdx.x), static_cast<int>(blockDim.x), 1};
  comm_run(task, blockIdx.x, gridDim.x, &scratch, g);
}

struct WaitList {
  const int* flags[COMM_MAX_WORLD];
  int n;
};

// One thread per flag waits (bounded) until the flag has reached `value`.  Placed in a stream in front of work that
// overwrites a buffer which peers may still be reading.
__global__ void wait_flags_kernel(const __grid_constant__ WaitList list, int value, int* status, long long wait_cycles) {
  const int p = threadIdx.x;
  if (p < list.n && list.flags[p] != nullptr)
    flag_wait_ge(list.flags[p], value, nullptr, status, wait_cycles > 0 ? wait_cycles : OB_WAIT_BUDGET_CYCLES);
}

__global__ void signal_kernel(int* flag, int value) {
  __threadfence_system();
  flag_store_release(flag, value);
}

// Layout of one rank's exchange area (symmetric memory): two parities x (8 values, 8 flags).
struct ScalarSlots {
  float vals[2][COMM_MAX_WORLD];
  int flags[2][COMM_MAX_WORLD];
};

// Every rank stores its value into slot [rank] of every peer, then waits until all of its own slots carry this epoch
// and sums them in rank order, so all ranks obtain the bit-identical total.  Returning from this kernel on every rank
// also implies that every rank has finished everything it enqueued before it.
__global__ void allreduce_scalar_kernel(const float* __restrict__ value, ScalarSlots* const* __restrict__ peers,
                                        ScalarSlots* mine, float* __restrict__ out, int rank, int world, int epoch,
                                        int* status, long long wait_cycles) {
  __shared__ int ok;
  const int par = epoch & 1;
  const int p = threadIdx.x;
  if (p == 0) ok = 1;
  __syncthreads();
  if (p < world) {
    ScalarSlots* dst = peers[p];
    dst->vals[par][rank] = *value;
    __threadfence_system();
    flag_store_release(&dst->flags[par][rank], epoch);
    if (!flag_wait_ge(&mine->flags[par][p], epoch, nullptr, status, wait_cycles > 0 ? wait_cycles : OB_WAIT_BUDGET_CYCLES)) ok = 0;
  }
  __syncthreads();
  if (p == 0) {
    float s = 0.f;
    if (ok) {
      for (int q = 0; q < world; ++q) s += *reinterpret_cast<volatile float*>(&mine->vals[par][q]);
    } else {
      s = *value;
    }
    out[0] = s;
  }
}

}  // namespace
}  // namespace ob

extern "C" int ob_comm_task_size(void) { return static_cast<int>(sizeof(ob::CommTask)); }

extern "C" int ob_comm_launch(const void* task, int nctas, cudaStream_t stream) {
  using namespace ob;
  const CommTask* t = reinterpret_cast<const CommTask*>(task);
  if (t == nullptr || t->world < 1 || t->world > COMM_MAX_WORLD || nctas < 1) return -1;
  if (t->kind == COMM_ALL_GATHER && (t->elems % 8 != 0)) return -2;
  if (t->kind == COMM_REDUCE_SCATTER && (t->elems % 4 != 0)) return -2;
  if (nctas > COMM_MAX_PARTS) return -1;
  comm_kernel<<<nctas, COMM_THREADS, 0, stream>>>(*t);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

// Waits until each of the `n` flags (device addresses, possibly in peers' memory; null entries are skipped) is >= value.
extern "C" int ob_wait_flags(const void* const* flags, int n, int value, int* status, long long wait_cycles,
                             cudaStream_t stream) {
  using namespace ob;
  if (n < 0 || n > COMM_MAX_WORLD) return -1;
  WaitList list = {};
  list.n = n;
  for (int i = 0; i < n; ++i) list.flags[i] = reinterpret_cast<const int*>(flags[i]);
  wait_flags_kernel<<<1, 32, 0, stream>>>(list, value, status, wait_cycles);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_signal(int* flag, int value, cudaStream_t stream) {
  ob::signal_kernel<<<1, 1, 0, stream>>>(flag, value);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_scalar_slots_bytes(void) { return static_cast<int>(sizeof(ob::ScalarSlots)); }

// `peers` is a device array of `world` pointers to every rank's exchange area (this rank's included).
extern "C" int ob_allreduce_scalar(const float* value, void* const* peers, void* mine, float* out, int rank, int world,
                                   int epoch, int* status, long long wait_cycles, cudaStream_t stream) {
  using namespace ob;
  if (world < 1 || world > COMM_MAX_WORLD) return -1;
  allreduce_scalar_kernel<<<1, 32, 0, stream>>>(value, reinterpret_cast<ScalarSlots* const*>(peers),
                                               reinterpret_cast<ScalarSlots*>(mine), out, rank, world, epoch, status, wait_cycles);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}
