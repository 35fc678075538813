// Shared pieces of the tcgen05 attention kernels (bf16): tile constants, the 4D TMA maps that read
// a [B, T, NH, D] or [B, NH, T, D] operand through its element strides, and the host-side checks
// of those strides.  The kernels work on 64-wide head tiles; a head_dim D < 64 (a multiple of 8)
// is served by the same kernels: the maps keep D as the tensor's inner extent with a 64-wide box,
// so TMA loads fill columns D..63 with zeros (which leaves Q K^T, P V and every gradient
// unchanged) and TMA stores clip them.
#pragma once

#include "tc_common.cuh"

namespace attn {

constexpr int AT_TILE = 128;                       // query / key rows per tile
constexpr int AT_D = 64;                           // head tile width of the tensor-core kernels (head_dim <= 64)
constexpr int AT_TILE_BYTES = AT_TILE * AT_D * 2;  // 16 KB bf16 tile, 128 B per row
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

struct TileMap {
  CUtensorMap map;
  int h_first;  // 1: dims {D, NH, T, B}; 0: dims {D, T, NH, B}
};

// 128 rows (t0 .. t0+127) of head h of batch b; rows past T read as zeros.
__device__ __forceinline__ void load_tile(void* dst, const TileMap& tm, uint64_t* bar, int b, int h,
                                          int t0) {
  if (tm.h_first)
    tma_load_4d(dst, &tm.map, bar, 0, h, t0, b);
  else
    tma_load_4d(dst, &tm.map, bar, 0, t0, h, b);
}

// Store a 128-row tile (swizzled like load_tile) from shared memory; rows past T are clipped.
__device__ __forceinline__ void store_tile(const TileMap& tm, const void* src, int b, int h, int t0) {
  if (tm.h_first)
    tma_store_4d(&tm.map, src, 0, h, t0, b);
  else
    tma_store_4d(&tm.map, src, 0, t0, h, b);
}

// head_dim values the tensor-core kernels serve: multiples of 8 (16-byte rows) up to the tile width.
inline bool tc_head_dim_ok(int D) { return D >= 8 && D <= AT_D && D % 8 == 0; }

// Element strides usable by TMA: 16-byte multiples and a row pitch of at least one head.
inline bool head_strides_ok(int64_t sb, int64_t st, int64_t sh, int D) {
  return sb % 8 == 0 && st % 8 == 0 && sh % 8 == 0 && st >= D;
}

// 4D map over a bf16 tensor with element (b, t, h, d) at base[b*sb + t*st + h*sh + d], d < D; the
// two middle dimensions are ordered by stride so the map's strides increase.  The box is always
// 64 wide in d (columns D..63 read as zeros, are not written).
inline bool make_head_map(TileMap* tm, const void* base, int B, int NH, int T, int D, int64_t sb,
                          int64_t st, int64_t sh) {
  uint64_t dims[4], strides[3];
  uint32_t box[4];
  tm->h_first = sh <= st ? 1 : 0;
  dims[0] = D;
  box[0] = AT_D;
  if (tm->h_first) {
    dims[1] = NH; dims[2] = T; dims[3] = B;
    strides[0] = sh * 2; strides[1] = st * 2; strides[2] = sb * 2;
    box[1] = 1; box[2] = AT_TILE; box[3] = 1;
  } else {
    dims[1] = T; dims[2] = NH; dims[3] = B;
    strides[0] = st * 2; strides[1] = sh * 2; strides[2] = sb * 2;
    box[1] = AT_TILE; box[2] = 1; box[3] = 1;
  }
  return make_tmap_bf16(&tm->map, base, 4, dims, strides, box);
}

// The same map over a float32 tensor (the tf32 path, head_dim <= 32): 128-byte rows of 32 elements,
// columns D..31 read as zeros.  swizzle_bytes selects the shared-memory layout (128, or
// SWIZZLE_128B_ATOM32 for operands the tf32 MMA reads MN-major).
inline bool make_head_map_f32(TileMap* tm, const void* base, int B, int NH, int T, int D, int64_t sb,
                              int64_t st, int64_t sh, int swizzle_bytes) {
  uint64_t dims[4], strides[3];
  uint32_t box[4];
  tm->h_first = sh <= st ? 1 : 0;
  dims[0] = D;
  box[0] = AT_D / 2;
  if (tm->h_first) {
    dims[1] = NH; dims[2] = T; dims[3] = B;
    strides[0] = sh * 4; strides[1] = st * 4; strides[2] = sb * 4;
    box[1] = 1; box[2] = AT_TILE; box[3] = 1;
  } else {
    dims[1] = T; dims[2] = NH; dims[3] = B;
    strides[0] = st * 4; strides[1] = sh * 4; strides[2] = sb * 4;
    box[1] = AT_TILE; box[2] = 1; box[3] = 1;
  }
  return make_tmap_f32(&tm->map, base, 4, dims, strides, box, swizzle_bytes);
}

// head_dim values of the tf32 tensor-core forward: multiples of 4 (16-byte rows) up to 32.
inline bool tc_head_dim_ok_tf32(int D) { return D >= 4 && D <= AT_D / 2 && D % 4 == 0; }

// Element strides usable by TMA for float32 tensors: 16-byte multiples.
inline bool head_strides_ok_f32(int64_t sb, int64_t st, int64_t sh, int D) {
  return sb % 4 == 0 && st % 4 == 0 && sh % 4 == 0 && st >= D;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Streaming multiprocessors of the current device (cached per device).
inline int current_device_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

// Per-device record of the CUDA context in which a one-time set-up step was done: a function
// attribute belongs to the module loaded in a context, so the step is redone in a new context
// (after a cudaDeviceReset).
struct CtxOnce {
  void* ctx[64] = {};
};

// Raise a kernel's dynamic shared-memory limit once per device and context.
template <typename Kernel>
inline bool set_smem_limit_once(Kernel kernel, int bytes, CtxOnce& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  void* ctx = current_context();
  if (ctx && done.ctx[dev] == ctx) return true;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(MaxDynamicSharedMemorySize=%d) failed: %s", bytes, cudaGetErrorString(e));
    return false;
  }
  done.ctx[dev] = current_context();
  return true;
}

// Whether `kernel` was built with the launch register allocation its setmaxnreg split was sized
// for (read once; `cached` holds it).  A kernel that moves registers between warpgroups must not
// launch otherwise: a warpgroup could wait for registers that never free up.
template <typename Kernel>
inline bool launch_regs_match(Kernel kernel, int expected, int& cached, const char* name) {
  if (cached == 0) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) {
      set_error("cudaFuncGetAttributes(%s) failed: %s", name, cudaGetErrorString(e));
      return false;
    }
    cached = fa.numRegs;
  }
  if (cached != expected) {
    set_error("%s: built with %d registers per thread, its register split needs %d", name, cached, expected);
    return false;
  }
  return true;
}

}  // namespace attn
