// Gradient all-reduce over NVSwitch multicast (NVLS) for data-parallel training.
//
// The reference trains on one GPU; its only scaling is gradient accumulation (auto_train.py:
// 1591-1615).  Here each rank's backward leaves its four parameter gradients in one flat float32
// buffer, and the ranks' buffers are summed (SUM, so every rank ends with the single-process
// full-batch gradient, model/gpt.py:687-694).  The buffer lives in symmetric memory bound to an
// NVLink multicast object (allocated by the caller, e.g. torch's symmetric memory): one virtual
// address (`mc`) whose loads and stores reach the buffer of every rank through the NVSwitch.
//
// Two-shot, in one kernel launch on every rank:
//   1. barrier: each block signals its counterpart block on every rank and waits for theirs, after
//      a system-scope fence, so every rank's gradients are complete and visible;
//   2. rank r owns 1/world of the buffer in 16-byte chunks: multimem.ld_reduce.add returns the sum
//      of a chunk over all ranks (the switch adds), multimem.st writes it back to every rank;
//   3. barrier again, so no rank reads its buffer before every slice has been written.
// Per GPU that moves about the buffer's size out and in over NVLink, with at most 128 small CTAs.
//
// The barriers use the caller's signal pads (one uint32 array per rank, all ranks' pads reachable
// by pointer): a signal sets a slot from 0 to 1 once its previous signal has been consumed, a wait
// consumes it (1 to 0), with system-scope atomics.  Every wait is bounded: after 2 s it records a
// site code in the library's status word (attn_device_error) and the kernel returns.
#include "tc_common.cuh"

namespace attn {

// 256 threads of at most 64 registers and no shared memory.  The reduction overlaps the GEMM that
// follows the weight gradients; that GEMM leaves it SMs of its own (attn_gemm_ex), since a block
// sharing an SM with a persistent GEMM CTA (192 threads of 255 registers) slows that CTA, and the
// GEMM ends with its slowest CTA.
constexpr int AR_THREADS = 256;
constexpr int AR_MAX_BLOCKS = 128;  // 2 channels x 128 blocks x 8 slots x 4 bytes = 8 KB of signal pad
constexpr int AR_MAX_WORLD = 8;     // ranks of one NVSwitch domain that one launch serves
constexpr int AR_UNROLL = 4;        // 16-byte chunks in flight per thread
constexpr uint64_t AR_WAIT_NS = 2000000000ull;
constexpr int AR_SITE_BARRIER_IN = 400, AR_SITE_BARRIER_OUT = 401;

__device__ __forceinline__ float4 mm_ld_reduce_add_v4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void mm_st_v4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float mm_ld_reduce_add(const float* mc) {
  float v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(v) : "l"(mc) : "memory");
  return v;
}

__device__ __forceinline__ void mm_st(float* mc, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}

// Set *slot from 0 to 1 (waiting until the previous signal has been consumed), bounded.
__device__ __forceinline__ bool ar_signal(uint32_t* slot, uint64_t t0) {
  while (atomicCAS_system(slot, 0u, 1u) != 0u) {
    if (globaltimer_ns() - t0 > AR_WAIT_NS) return false;
    __nanosleep(64);
  }
  return true;
}

// Consume a signal: *slot from 1 to 0 (waiting until it is set), bounded.
__device__ __forceinline__ bool ar_consume(uint32_t* slot, uint64_t t0) {
  while (atomicCAS_system(slot, 1u, 0u) != 1u) {
    if (globaltimer_ns() - t0 > AR_WAIT_NS) return false;
    __nanosleep(64);
  }
  return true;
}

// Block b of this rank meets block b of every rank.  Slot (channel, b, s) of rank p's pad is set
// by rank s.  Thread t < world handles peer t.  Returns false (after recording `site`) if a wait
// gave up; uniform over the block.
__device__ __forceinline__ bool ar_barrier(uint32_t* const* pads, int rank, int world, int channel,
                                           const WaitErr& werr, int site) {
  __syncthreads();
  bool ok = true;
  if (threadIdx.x < (unsigned)world) {
    const int peer = threadIdx.x;
    const size_t base = ((size_t)channel * gridDim.x + blockIdx.x) * AR_MAX_WORLD;
    __threadfence_system();  // this rank's writes (earlier kernels, this block) before the signal
    const uint64_t t0 = globaltimer_ns();
    ok = ar_signal(pads[peer] + base + rank, t0) && ar_consume(pads[rank] + base + peer, t0);
    __threadfence_system();  // the peers' writes before what follows
    if (!ok) record_wait_error(werr, site);
  }
  return __syncthreads_and(ok) != 0;
}

__global__ void __launch_bounds__(AR_THREADS, 4)  // at most 64 registers per thread
grad_allreduce_kernel(float* __restrict__ mc, uint32_t* const* __restrict__ pads, int rank, int world, int64_t n,
                      int* err) {
  const WaitErr werr = wait_err(err);
  if (!ar_barrier(pads, rank, world, 0, werr, AR_SITE_BARRIER_IN)) return;
  // this rank's slice of the 16-byte chunks
  const int64_t n4 = n / 4;
  const int64_t per = (n4 + world - 1) / world;
  const int64_t lo = min(n4, per * rank), hi = min(n4, lo + per);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < hi; i0 += stride * AR_UNROLL) {
    float4 v[AR_UNROLL];
#pragma unroll
    for (int u = 0; u < AR_UNROLL; ++u)
      if (i0 + u * stride < hi) v[u] = mm_ld_reduce_add_v4(mc + 4 * (i0 + u * stride));
#pragma unroll
    for (int u = 0; u < AR_UNROLL; ++u)
      if (i0 + u * stride < hi) mm_st_v4(mc + 4 * (i0 + u * stride), v[u]);
  }
  // the n % 4 trailing floats: the last rank's first block
  if (rank == world - 1 && blockIdx.x == 0 && threadIdx.x < (unsigned)(n & 3)) {
    float* p = mc + 4 * n4 + threadIdx.x;
    mm_st(p, mm_ld_reduce_add(p));
  }
  ar_barrier(pads, rank, world, 1, werr, AR_SITE_BARRIER_OUT);
}

// Blocks of one launch, the same count on every rank (the barrier pairs blocks by index): no more
// than the slice needs, at most max_blocks (0: AR_DEFAULT_BLOCKS).  Sixteen reach the NVSwitch
// rate on 8 GPUs (42 us for 9.45 MB back to back, as 128 do) and need only the 16 SMs that the
// GEMM beside the reduction leaves free.
constexpr int AR_DEFAULT_BLOCKS = 16;
static int ar_blocks(int64_t n, int world, int max_blocks) {
  const int64_t per_rank = (n / 4 + world - 1) / world;
  int64_t b = (per_rank + (int64_t)AR_THREADS * AR_UNROLL - 1) / ((int64_t)AR_THREADS * AR_UNROLL);
  const int cap = max_blocks > 0 ? (max_blocks < AR_MAX_BLOCKS ? max_blocks : AR_MAX_BLOCKS) : AR_DEFAULT_BLOCKS;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace attn

extern "C" size_t attn_grad_allreduce_signal_bytes(int64_t n, int world) {
  using namespace attn;
  if (n <= 0 || world < 1) return 0;
  return (size_t)2 * AR_MAX_BLOCKS * AR_MAX_WORLD * sizeof(uint32_t);  // enough for any block count
}

extern "C" int attn_grad_allreduce(void* multicast, const void* signal_pads, int rank, int world, int64_t n,
                                   size_t signal_pad_bytes, int max_blocks, void* stream) {
  using namespace attn;
  clear_error();
  ATTN_REQUIRE(multicast && signal_pads, "attn_grad_allreduce: null pointer argument");
  ATTN_REQUIRE(world >= 2 && world <= AR_MAX_WORLD, "attn_grad_allreduce: world size %d outside 2 .. %d", world,
               AR_MAX_WORLD);
  ATTN_REQUIRE(rank >= 0 && rank < world, "attn_grad_allreduce: rank %d outside the world of %d", rank, world);
  ATTN_REQUIRE(n > 0, "attn_grad_allreduce: the buffer must hold at least one float");
  ATTN_REQUIRE(aligned(multicast, 16), "attn_grad_allreduce: the multicast address must be 16-byte aligned");
  const size_t need = attn_grad_allreduce_signal_bytes(n, world);
  ATTN_REQUIRE(signal_pad_bytes >= need, "attn_grad_allreduce: signal pads of %zu bytes needed, %zu given", need,
               signal_pad_bytes);
  int* err = dev_error_ptr();
  if (!err) return ATTN_ERR_CUDA;
  ATTN_REQUIRE(max_blocks >= 0, "attn_grad_allreduce: max_blocks must be >= 0");
  grad_allreduce_kernel<<<ar_blocks(n, world, max_blocks), AR_THREADS, 0, as_stream(stream)>>>(
      static_cast<float*>(multicast), static_cast<uint32_t* const*>(signal_pads), rank, world, n, err);
  count_launch();
  return check_launch("grad_allreduce_kernel");
}
