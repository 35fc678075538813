// Single-query decode attention: one new query row per (b, h) over an L-token K/V prefix.
//
// The reference has no KV cache: GenerationSession.generate re-runs the full causal forward for
// every new token and keeps only the last row (generate.py:611-628).  This kernel computes that
// last row directly from a cache.  The work is a pure stream over K and V (2*L*D elements per
// (b, h)), so it is bound by HBM bandwidth: the L axis is split across CTAs (flash-decoding),
// each CTA writes an unnormalised partial softmax state (m, l, o[D]) to the workspace, and a
// second kernel merges the splits.
//
// Lane layout: a key row of D elements is read by LPK = D / EPL lanes, each loading one 16-byte
// vector (EPL = 8 bf16 or 4 fp32 elements); a warp therefore reads KPW = 32 / LPK keys per step,
// each lane group keeps its own online-softmax state, and the states are merged at the end.
#include "tc_common.cuh"
#include <math.h>

namespace attn {

constexpr int DEC_THREADS = 128;
constexpr int DEC_CHUNK = 256;  // keys per split

static int decode_splits(int L) { return (L + DEC_CHUNK - 1) / DEC_CHUNK; }

size_t decode_ws(int B, int NH, int L, int D) {
  return (size_t)B * NH * decode_splits(L) * (D + 2) * sizeof(float);
}

// The partial kernel runs one grid row per (b, h): B*NH is its grid.y, at most 65535.
int decode_grid_check(int B, int NH, const char* fn) {
  if ((int64_t)B * NH > 65535) {
    set_error("%s: B*NH = %lld (sequences x heads) exceeds the decode kernel's limit of 65535; split the "
              "batch into several calls", fn, (long long)B * NH);
    return ATTN_ERR_UNSUPPORTED;
  }
  return ATTN_OK;
}

template <typename T> struct Vec16;
template <> struct Vec16<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void load(const float* p, float* out) {
    float4 v = *reinterpret_cast<const float4*>(p);
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  }
};
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* out) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      float2 f = __bfloat1622float2(h);
      out[2 * i] = f.x;
      out[2 * i + 1] = f.y;
    }
  }
};

template <typename T, int D>
__global__ void __launch_bounds__(DEC_THREADS)
attn_decode_partial_kernel(const T* __restrict__ q, const T* __restrict__ kc,
                           const T* __restrict__ vc, float* __restrict__ ws, int NH, int L,
                           int64_t q_sb, int64_t q_sh, int64_t kv_sb, int64_t kv_sl,
                           int64_t kv_sh, float scale) {
  constexpr int EPL = Vec16<T>::N;
  constexpr int LPK = D / EPL;            // lanes per key
  constexpr int KPW = 32 / LPK;           // keys per warp step
  constexpr int NW = DEC_THREADS / 32;
  constexpr int NSTATE = NW * KPW;
  static_assert(D % EPL == 0 && LPK <= 32, "unsupported head_dim for decode");
  __shared__ float sm_m[NSTATE], sm_l[NSTATE];
  __shared__ float sm_o[NSTATE][D];

  const int bh = blockIdx.y, b = bh / NH, h = bh % NH;
  const int split = blockIdx.x, nsplit = gridDim.x;
  const int l0 = split * DEC_CHUNK, l1 = min(L, l0 + DEC_CHUNK);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int grp = lane / LPK, sub = lane % LPK;

  float qf[EPL];
  Vec16<T>::load(q + b * q_sb + h * q_sh + sub * EPL, qf);
#pragma unroll
  for (int i = 0; i < EPL; ++i) qf[i] *= scale;
  const T* kb = kc + b * kv_sb + h * kv_sh + sub * EPL;
  const T* vb = vc + b * kv_sb + h * kv_sh + sub * EPL;

  float m = -INFINITY, lsum = 0.f, acc[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) acc[i] = 0.f;

  for (int base = l0 + warp * KPW; base < l1; base += NW * KPW) {
    const int key = base + grp;
    const bool valid = key < l1;
    float kf[EPL], vf[EPL];
    float s = 0.f;
    if (valid) {
      Vec16<T>::load(kb + key * kv_sl, kf);
      Vec16<T>::load(vb + key * kv_sl, vf);
#pragma unroll
      for (int i = 0; i < EPL; ++i) s += qf[i] * kf[i];
    }
#pragma unroll
    for (int off = LPK / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (valid) {
      const float m_new = fmaxf(m, s);
      const float corr = expf(m - m_new);
      const float p = expf(s - m_new);
      lsum = lsum * corr + p;
#pragma unroll
      for (int i = 0; i < EPL; ++i) acc[i] = acc[i] * corr + p * vf[i];
      m = m_new;
    }
  }
  const int state = warp * KPW + grp;
  if (sub == 0) {
    sm_m[state] = m;
    sm_l[state] = lsum;
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) sm_o[state][sub * EPL + i] = acc[i];
  __syncthreads();

  float M = -INFINITY;
  for (int i = 0; i < NSTATE; ++i) M = fmaxf(M, sm_m[i]);
  float* out = ws + ((int64_t)bh * nsplit + split) * (D + 2);
  for (int d = threadIdx.x; d < D; d += DEC_THREADS) {
    float o = 0.f;
    for (int i = 0; i < NSTATE; ++i)
      if (sm_m[i] != -INFINITY) o += sm_o[i][d] * expf(sm_m[i] - M);
    out[2 + d] = o;
  }
  if (threadIdx.x == 0) {
    float l = 0.f;
    for (int i = 0; i < NSTATE; ++i)
      if (sm_m[i] != -INFINITY) l += sm_l[i] * expf(sm_m[i] - M);
    out[0] = M;
    out[1] = l;
  }
}

template <typename T, int D>
__global__ void attn_decode_combine_kernel(const float* __restrict__ ws, int nsplit, int NH,
                                           T* __restrict__ o, float* __restrict__ lse,
                                           int64_t q_sb, int64_t q_sh) {
  const int bh = blockIdx.x, b = bh / NH, h = bh % NH;
  const float* st = ws + (int64_t)bh * nsplit * (D + 2);
  float M = -INFINITY;
  for (int i = 0; i < nsplit; ++i) M = fmaxf(M, st[i * (D + 2)]);
  float l = 0.f;
  for (int i = 0; i < nsplit; ++i) l += st[i * (D + 2) + 1] * expf(st[i * (D + 2)] - M);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < nsplit; ++i) acc += st[i * (D + 2) + 2 + d] * expf(st[i * (D + 2)] - M);
    Elem<T>::store(o + b * q_sb + h * q_sh + d, acc / l);
  }
  if (threadIdx.x == 0 && lse) lse[bh] = M + logf(l);
}

template <typename T, int D>
static int decode_d(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH,
                    int L, int64_t q_sb, int64_t q_sh, int64_t kv_sb, int64_t kv_sl, int64_t kv_sh,
                    float scale, float* ws, cudaStream_t s) {
  const int ns = decode_splits(L);
  dim3 g1(ns, B * NH);
  attn_decode_partial_kernel<T, D><<<g1, DEC_THREADS, 0, s>>>((const T*)q, (const T*)k, (const T*)v,
      ws, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale);
  count_launch();
  int rc = check_launch("attn_decode_partial_kernel");
  if (rc) return rc;
  attn_decode_combine_kernel<T, D><<<B * NH, D < 32 ? 32 : D, 0, s>>>(ws, ns, NH, (T*)o, lse, q_sb,
                                                                      q_sh);
  count_launch();
  return check_launch("attn_decode_combine_kernel");
}

int decode(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH, int L,
           int D, int64_t q_sb, int64_t q_sh, int64_t kv_sb, int64_t kv_sl, int64_t kv_sh,
           float scale, int dtype, float* ws, cudaStream_t s) {
  if (dtype == ATTN_BF16) {
    switch (D) {
      case 8: return decode_d<__nv_bfloat16, 8>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 16: return decode_d<__nv_bfloat16, 16>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 32: return decode_d<__nv_bfloat16, 32>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 64: return decode_d<__nv_bfloat16, 64>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 128: return decode_d<__nv_bfloat16, 128>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
    }
  } else {
    switch (D) {
      case 4: return decode_d<float, 4>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 8: return decode_d<float, 8>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 16: return decode_d<float, 16>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 32: return decode_d<float, 32>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 64: return decode_d<float, 64>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
      case 128: return decode_d<float, 128>(q, k, v, o, lse, B, NH, L, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale, ws, s);
    }
  }
  set_error("attn_decode: head_dim %d not supported for this dtype", D);
  return ATTN_ERR_UNSUPPORTED;
}

}  // namespace attn

// ------------------------------------------------------------------------------------------
// attn_decode_noalloc: the same decode with its scratch in a fixed device array
// ------------------------------------------------------------------------------------------
// Some callers cannot hand this library a workspace: their device memory belongs to another
// allocator (a pool that reserved the free HBM up front, as the reference's monkey-patched
// pycuda mem_alloc pool or a serving process that pre-sizes its KV cache does), or they are thin
// FFI callers that hold only the q/K/V/o pointers.  For them the per-split partial softmax
// states live in this file-scope array, sized once at load time; every GPU that loads the
// library holds it until the process exits.
namespace attn {

constexpr size_t kNoAllocDecodeFloats = size_t(1) << 20;  // 4 MiB
static __device__ __align__(256) float g_decode_scratch[kNoAllocDecodeFloats];
static SymbolCache g_decode_scratch_cache;

// The array's device address on the current device, resolved on the first call per device (and
// again if the device's CUDA context changes, since the module then reloads).
static float* decode_scratch_address() {
  return static_cast<float*>(device_symbol_address(g_decode_scratch_cache, (const void*)&g_decode_scratch,
                                                   "attn_decode_noalloc"));
}

}  // namespace attn

extern "C" int attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* o,
                                   float* lse, int B, int NH, int L, int D, int64_t q_sb,
                                   int64_t q_sh, int64_t kv_sb, int64_t kv_sl, int64_t kv_sh,
                                   float scale, int dtype, void* stream) {
  using namespace attn;
  clear_error();
  ATTN_REQUIRE(q && k_cache && v_cache && o, "attn_decode_noalloc: null pointer argument");
  ATTN_REQUIRE(dtype == ATTN_F32 || dtype == ATTN_BF16, "attn_decode_noalloc: bad dtype");
  ATTN_REQUIRE(B > 0 && NH > 0 && L > 0 && D > 0, "attn_decode_noalloc: sizes must be positive");
  const int vec = dtype == ATTN_F32 ? 4 : 8;
  ATTN_REQUIRE(D % vec == 0, "attn_decode_noalloc: head_dim must be a multiple of %d for this dtype", vec);
  const int64_t st[5] = {q_sb, q_sh, kv_sb, kv_sl, kv_sh};
  for (int i = 0; i < 5; ++i)
    ATTN_REQUIRE(st[i] >= 0 && st[i] % vec == 0, "attn_decode_noalloc: strides must be multiples of %d", vec);
  ATTN_REQUIRE(aligned(q, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(o, 4),
               "attn_decode_noalloc: q/k/v must be 16-byte aligned");
  if (int rc = decode_grid_check(B, NH, "attn_decode_noalloc")) return rc;
  const size_t need = decode_ws(B, NH, L, D);
  if (need > sizeof(float) * kNoAllocDecodeFloats) {
    set_error("attn_decode_noalloc: this problem needs %zu bytes of scratch but the fixed array holds "
              "%zu (B*NH*ceil(L/256)*(D+2) must be <= %zu floats); use attn_decode with a workspace",
              need, sizeof(float) * kNoAllocDecodeFloats, kNoAllocDecodeFloats);
    return ATTN_ERR_UNSUPPORTED;
  }
  float* ws = decode_scratch_address();
  if (!ws) return ATTN_ERR_CUDA;
  // every partial state is written before it is read: nothing in the array needs zeroing
  return decode(q, k_cache, v_cache, o, lse, B, NH, L, D, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale,
                dtype, ws, as_stream(stream));
}
