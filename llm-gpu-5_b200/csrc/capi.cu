// extern "C" entry points of libattn_b200.so (declared in include/attn_b200.h).
//
// Every entry point validates its arguments before launching anything: a null pointer, a bad
// shape, a misaligned or inconsistent stride, or a short workspace returns a negative code and
// sets the per-thread error string; no kernel runs.  This mirrors the reference's failure
// behaviour at the API level (MultiHeadAttention raises before touching the GPU when its caches
// are missing, model/gpt.py:649-650) while keeping the ABI free of exceptions.
#include "tc_common.cuh"

#include <atomic>
#include <mutex>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

namespace attn {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}
void clear_error() { g_last_error.clear(); }
void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return ATTN_ERR_CUDA;
  }
  return ATTN_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("ATTN_NO_PDL");
    return !(v && v[0] && strcmp(v, "0") != 0);
  }();
  return on;
}

int check_launch(const char* what, cudaError_t launched) {
  const cudaError_t last = cudaGetLastError();  // read (and clear) the runtime's record either way
  const cudaError_t e = launched != cudaSuccess ? launched : last;
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return ATTN_ERR_CUDA;
  }
  return ATTN_OK;
}

// ---- CUDA context of the calling thread (driver API through the runtime's entry point) --------
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

void* current_context() {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  CUcontext c = nullptr;
  if (fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

static std::mutex g_symbol_mu;

void* device_symbol_address(SymbolCache& cache, const void* symbol, const char* what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("%s: cudaGetDevice failed: %s", what, cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_symbol_mu);
  void* ctx = current_context();
  if (cache.ptr[dev] && ctx && cache.ctx[dev] == ctx) return cache.ptr[dev];
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, symbol);  // creates the primary context if there is none yet
  if (e != cudaSuccess || p == nullptr) {
    set_error("%s: cudaGetSymbolAddress failed on device %d: %s", what, dev, cudaGetErrorString(e));
    return nullptr;
  }
  cache.ctx[dev] = current_context();
  cache.ptr[dev] = p;
  return p;
}

// ---- device error word pair of the tensor-core kernels' bounded waits ------------------------
// [0]: site code of the first wait that gave up since the last clear; [1]: give-ups, ever.
static __device__ int g_dev_error[2];
static SymbolCache g_dev_error_cache;

int* dev_error_ptr() {
  return static_cast<int*>(device_symbol_address(g_dev_error_cache, (const void*)&g_dev_error,
                                                 "device error word"));
}

// ---- TMA tensor maps through the driver entry point (no libcuda link dependency) ----------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

static bool make_tmap(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int rank,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable");
    return false;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i < rank - 1) st[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dt, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_bytes == 64                    ? CU_TENSOR_MAP_SWIZZLE_64B
                  : swizzle_bytes == SWIZZLE_128B_ATOM32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                         : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): rank %d dims %llu x %llu", (int)r, rank,
              (unsigned long long)dims[0], (unsigned long long)dims[1]);
    return false;
  }
  return true;
}

bool make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  return make_tmap(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides_bytes, box, swizzle_bytes);
}

bool make_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  return make_tmap(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, rank, dims, strides_bytes, box, swizzle_bytes);
}

static int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// implemented in the kernel translation units
int attn_fwd_simt(const void*, const void*, const void*, void*, float*, int, int, int, int,
                  const int64_t*, float, int, cudaStream_t);
int attn_bwd_simt(const void*, const void*, const void*, const void*, const void*, const float*,
                  void*, void*, void*, float*, int, int, int, int, const int64_t*, float, int,
                  cudaStream_t);
int gemm_simt(const void*, int64_t, int, const void*, int64_t, int, int, void*, int64_t, int,
              const float*, int, int, int, int, cudaStream_t, int act = ACT_NONE, void* aux = nullptr,
              int64_t ldaux = 0, int aux_dtype = ATTN_F32);
int split_heads(const float*, float*, float*, float*, int, int, int, int, cudaStream_t);
int merge_heads(const float*, float*, int, int, int, int, cudaStream_t);
int cast_f32_bf16(const float*, void*, int64_t, cudaStream_t, int);
int cast_rows_ones(const float*, int64_t, int, int, void*, int64_t, cudaStream_t, int);
int layernorm_rows(const float*, int64_t, const float*, const float*, int, int, float, void*, int64_t, int, int,
                   cudaStream_t);
int layernorm_bwd_rows(const float*, const float*, const float*, int, int, float, float*, int, float*, float*, int,
                       cudaStream_t, int);
size_t colsum_ws(int, int);
int colsum(const void*, int, int64_t, int, int, float*, int, void*, cudaStream_t);
int cast_colsum(const float*, int64_t, int, int, void*, int64_t, float*, int, void*, cudaStream_t);
int attn_probs_launch(const void*, const void*, const float*, float*, int, int, int, int, int64_t,
                      int64_t, int64_t, float, int, cudaStream_t);
size_t decode_ws(int, int, int, int);
int decode_grid_check(int, int, const char*);
int wait_selftest(int, cudaStream_t);
int decode(const void*, const void*, const void*, void*, float*, int, int, int, int, int64_t,
           int64_t, int64_t, int64_t, int64_t, float, int, float*, cudaStream_t);
bool tc_fwd_supported(int D, int dtype);
bool tc_attn_layout_ok(const void* const* ptrs, int n, const int64_t* s, int D, int esz);
int attn_fwd_tc(const void*, const void*, const void*, void*, float*, int, int, int, int,
                const int64_t*, float, cudaStream_t, int tf32);
bool tc_bwd_supported(int D, int T, int dtype);
size_t attn_bwd_tc_ws(int B, int NH, int T, int D);
int attn_bwd_tc(const void*, const void*, const void*, const void*, const void*, const float*,
                void*, void*, void*, void*, int, int, int, int, const int64_t*, float,
                cudaStream_t);
bool tc_gemm_supported(int M, int N, int K, int64_t lda, int a_trans, int64_t ldb, int b_trans,
                       const void* A, const void* B, int tf32);
int gemm_tc(const void*, int64_t, int, const void*, int64_t, int, void*, int64_t, int,
            const float*, int, int, int, int, cudaStream_t, int act = ACT_NONE, const void* aux = nullptr,
            int64_t ldaux = 0, int aux_dtype = ATTN_F32, int tf32 = 0, int max_ctas = 0);
bool tc_gemm_act_ok(const void* C, int64_t ldc, int c_dtype, int act, const void* aux, int64_t ldaux,
                    int aux_dtype);

static size_t elem_size(int dtype) { return dtype == ATTN_BF16 ? 2 : 4; }

// The attention kernels' arithmetic for a storage type: ATTN_TF32 operands are float32 storage, and
// the attention kernels serve them with their float32 arithmetic.
static int attn_arith(int dtype) { return dtype == ATTN_TF32 ? ATTN_F32 : dtype; }

static int check_attn_args(const char* fn, int B, int NH, int T, int D, int dtype,
                           const int64_t* st) {
  ATTN_REQUIRE(dtype == ATTN_F32 || dtype == ATTN_BF16, "%s: dtype must be ATTN_F32 or ATTN_BF16", fn);
  ATTN_REQUIRE(B > 0 && NH > 0 && T > 0 && D > 0, "%s: B, NH, T, D must be positive (got %d %d %d %d)",
               fn, B, NH, T, D);
  ATTN_REQUIRE(D % 4 == 0, "%s: head_dim %d must be a multiple of 4", fn, D);
  for (int i = 0; i < 6; ++i)
    ATTN_REQUIRE(st[i] >= 0 && st[i] % 4 == 0,
                 "%s: strides must be non-negative multiples of 4 elements (stride %d = %lld)", fn, i,
                 (long long)st[i]);
  ATTN_REQUIRE(st[1] >= D && st[4] >= D, "%s: row strides must be >= head_dim", fn);
  return ATTN_OK;
}

}  // namespace attn

using namespace attn;

extern "C" {

int attn_version(void) { return 100; }

const char* attn_last_error_string(void) { return g_last_error.c_str(); }

uint64_t attn_launch_count(void) { return g_launches.load(); }

int attn_device_error(int clear) {
  clear_error();
  int* p = dev_error_ptr();
  if (!p) return ATTN_ERR_CUDA;
  int v = 0;
  ATTN_CUDA_TRY(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear && v) {
    const int z = 0;
    ATTN_CUDA_TRY(cudaMemcpy(p, &z, sizeof(int), cudaMemcpyHostToDevice));
  }
  return v;
}

int attn_device_error_async(int* host_dst, void* stream) {
  clear_error();
  ATTN_REQUIRE(host_dst, "attn_device_error_async: null destination");
  int* p = dev_error_ptr();
  if (!p) return ATTN_ERR_CUDA;
  ATTN_CUDA_TRY(cudaMemcpyAsync(host_dst, p, sizeof(int), cudaMemcpyDeviceToHost, as_stream(stream)));
  return ATTN_OK;
}

int attn_wait_selftest(int limit_us, void* stream) {
  clear_error();
  ATTN_REQUIRE(limit_us >= 1 && limit_us <= 1000000, "attn_wait_selftest: limit_us must be 1 .. 1000000");
  return wait_selftest(limit_us, as_stream(stream));
}

int attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH, int T,
             int D, int64_t in_sb, int64_t in_st, int64_t in_sh, int64_t out_sb, int64_t out_st,
             int64_t out_sh, float scale, int dtype, void* stream) {
  clear_error();
  const int requested = dtype;  // ATTN_TF32 selects the tf32 tensor-core forward where it applies
  dtype = attn_arith(dtype);
  ATTN_REQUIRE(q && k && v && o && lse, "attn_fwd: null pointer argument");
  const int64_t st[6] = {in_sb, in_st, in_sh, out_sb, out_st, out_sh};
  if (int rc = check_attn_args("attn_fwd", B, NH, T, D, dtype, st)) return rc;
  const size_t a = 4 * elem_size(dtype);
  ATTN_REQUIRE(aligned(q, a) && aligned(k, a) && aligned(v, a) && aligned(o, a),
               "attn_fwd: q/k/v/o must be %zu-byte aligned", a);
  const void* tens[4] = {q, k, v, o};
  // tensor-core path for bf16 head_dim <= 64 whenever the layout suits TMA; CUDA cores otherwise
  if (tc_fwd_supported(D, requested) && tc_attn_layout_ok(tens, 4, st, D, (int)elem_size(dtype)))
    return attn_fwd_tc(q, k, v, o, lse, B, NH, T, D, st, scale, as_stream(stream), requested == ATTN_TF32);
  return attn_fwd_simt(q, k, v, o, lse, B, NH, T, D, st, scale, dtype, as_stream(stream));
}

size_t attn_bwd_workspace_size(int B, int NH, int T, int D, int dtype) {
  dtype = attn_arith(dtype);
  if (B <= 0 || NH <= 0 || T <= 0 || D <= 0) return 0;
  size_t ws = (size_t)B * NH * T * sizeof(float);  // delta = rowsum(dO * O)
  if (tc_bwd_supported(D, T, dtype)) ws = attn_bwd_tc_ws(B, NH, T, D);
  return ws;
}

int attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
             const float* lse, void* dq, void* dk, void* dv, void* workspace,
             size_t workspace_bytes, int B, int NH, int T, int D, int64_t in_sb, int64_t in_st,
             int64_t in_sh, int64_t out_sb, int64_t out_st, int64_t out_sh, float scale, int dtype,
             void* stream) {
  clear_error();
  const int requested = dtype;  // ATTN_TF32: scores recomputed from tf32 q and k (see attn_bwd_simt)
  dtype = attn_arith(dtype);
  ATTN_REQUIRE(q && k && v && o && dout && lse && dq && dk && dv, "attn_bwd: null pointer argument");
  const int64_t st[6] = {in_sb, in_st, in_sh, out_sb, out_st, out_sh};
  if (int rc = check_attn_args("attn_bwd", B, NH, T, D, dtype, st)) return rc;
  const size_t need = attn_bwd_workspace_size(B, NH, T, D, dtype);
  if (!workspace || workspace_bytes < need) {
    set_error("attn_bwd: workspace of %zu bytes required, %zu given", need,
              workspace ? workspace_bytes : (size_t)0);
    return ATTN_ERR_WORKSPACE;
  }
  ATTN_REQUIRE(aligned(workspace, 256), "attn_bwd: workspace must be 256-byte aligned");
  const size_t a = 4 * elem_size(dtype);
  ATTN_REQUIRE(aligned(q, a) && aligned(k, a) && aligned(v, a) && aligned(o, a) && aligned(dout, a) &&
                   aligned(dq, a) && aligned(dk, a) && aligned(dv, a),
               "attn_bwd: tensors must be %zu-byte aligned", a);
  const void* tens[8] = {q, k, v, o, dout, dq, dk, dv};
  // the tensor-core workspace (attn_bwd_workspace_size) also covers the CUDA-core path
  if (tc_bwd_supported(D, T, dtype) && tc_attn_layout_ok(tens, 8, st, D, 2))
    return attn_bwd_tc(q, k, v, o, dout, lse, dq, dk, dv, workspace, B, NH, T, D, st, scale,
                       as_stream(stream));
  return attn_bwd_simt(q, k, v, o, dout, lse, dq, dk, dv, (float*)workspace, B, NH, T, D, st, scale,
                       requested, as_stream(stream));
}

int attn_probs(const void* q, const void* k, const float* lse, float* probs, int B, int NH, int T,
               int D, int64_t in_sb, int64_t in_st, int64_t in_sh, float scale, int dtype,
               void* stream) {
  clear_error();
  dtype = attn_arith(dtype);
  ATTN_REQUIRE(q && k && lse && probs, "attn_probs: null pointer argument");
  ATTN_REQUIRE(dtype == ATTN_F32 || dtype == ATTN_BF16, "attn_probs: bad dtype");
  ATTN_REQUIRE(B > 0 && NH > 0 && T > 0 && D > 0, "attn_probs: sizes must be positive");
  ATTN_REQUIRE(in_sb >= 0 && in_st >= D && in_sh >= 0, "attn_probs: bad strides");
  return attn_probs_launch(q, k, lse, probs, B, NH, T, D, in_sb, in_st, in_sh, scale, dtype,
                           as_stream(stream));
}

size_t attn_decode_workspace_size(int B, int NH, int L, int D) {
  if (B <= 0 || NH <= 0 || L <= 0 || D <= 0) return 0;
  return decode_ws(B, NH, L, D);
}

int attn_decode(const void* q, const void* k_cache, const void* v_cache, void* o, float* lse, int B,
                int NH, int L, int D, int64_t q_sb, int64_t q_sh, int64_t kv_sb, int64_t kv_sl,
                int64_t kv_sh, float scale, int dtype, void* workspace, size_t workspace_bytes,
                void* stream) {
  clear_error();
  ATTN_REQUIRE(q && k_cache && v_cache && o, "attn_decode: null pointer argument");
  ATTN_REQUIRE(dtype == ATTN_F32 || dtype == ATTN_BF16, "attn_decode: bad dtype");
  ATTN_REQUIRE(B > 0 && NH > 0 && L > 0 && D > 0, "attn_decode: sizes must be positive");
  const int vec = 16 / (int)elem_size(dtype);
  ATTN_REQUIRE(D % vec == 0, "attn_decode: head_dim must be a multiple of %d for this dtype", vec);
  const int64_t st[5] = {q_sb, q_sh, kv_sb, kv_sl, kv_sh};
  for (int i = 0; i < 5; ++i)
    ATTN_REQUIRE(st[i] >= 0 && st[i] % vec == 0, "attn_decode: strides must be multiples of %d", vec);
  ATTN_REQUIRE(aligned(q, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(o, 4),
               "attn_decode: q/k/v must be 16-byte aligned");
  if (int rc = decode_grid_check(B, NH, "attn_decode")) return rc;
  const size_t need = decode_ws(B, NH, L, D);
  if (!workspace || workspace_bytes < need) {
    set_error("attn_decode: workspace of %zu bytes required", need);
    return ATTN_ERR_WORKSPACE;
  }
  return decode(q, k_cache, v_cache, o, lse, B, NH, L, D, q_sb, q_sh, kv_sb, kv_sl, kv_sh, scale,
                dtype, (float*)workspace, as_stream(stream));
}

int attn_gemm(const void* A, int64_t lda, int a_trans, const void* B, int64_t ldb, int b_trans,
              int ab_dtype, void* C, int64_t ldc, int c_dtype, const float* bias, int M, int N, int K,
              int accumulate, void* stream) {
  return attn_gemm_ex(A, lda, a_trans, B, ldb, b_trans, ab_dtype, C, ldc, c_dtype, bias, M, N, K, accumulate, 0,
                      stream);
}

int attn_gemm_ex(const void* A, int64_t lda, int a_trans, const void* B, int64_t ldb, int b_trans,
                 int ab_dtype, void* C, int64_t ldc, int c_dtype, const float* bias, int M, int N, int K,
                 int accumulate, int max_ctas, void* stream) {
  clear_error();
  ATTN_REQUIRE(max_ctas >= 0, "attn_gemm: max_ctas must be >= 0");
  ATTN_REQUIRE(A && B && C, "attn_gemm: null pointer argument");
  ATTN_REQUIRE(M > 0 && N > 0 && K > 0, "attn_gemm: M, N, K must be positive");
  ATTN_REQUIRE(ab_dtype == ATTN_F32 || ab_dtype == ATTN_BF16 || ab_dtype == ATTN_TF32,
               "attn_gemm: bad operand dtype");
  ATTN_REQUIRE(c_dtype == ATTN_F32 || c_dtype == ATTN_BF16, "attn_gemm: bad output dtype");
  ATTN_REQUIRE(!accumulate || c_dtype == ATTN_F32, "attn_gemm: accumulate requires a float32 C");
  ATTN_REQUIRE(lda >= (a_trans ? M : K) && ldb >= (b_trans ? K : N) && ldc >= N,
               "attn_gemm: leading dimensions too small");
  const int tf32 = ab_dtype == ATTN_TF32;
  if (ab_dtype != ATTN_F32 && tc_gemm_supported(M, N, K, lda, a_trans, ldb, b_trans, A, B, tf32))
    return gemm_tc(A, lda, a_trans, B, ldb, b_trans, C, ldc, c_dtype, bias, M, N, K, accumulate,
                   as_stream(stream), ACT_NONE, nullptr, 0, ATTN_F32, tf32, max_ctas);
  // shapes the tensor-core kernel does not take: tf32 operands are float32 storage, so the exact
  // float32 CUDA-core GEMM serves them
  return gemm_simt(A, lda, a_trans, B, ldb, b_trans, tf32 ? ATTN_F32 : ab_dtype, C, ldc, c_dtype, bias, M, N,
                   K, accumulate, as_stream(stream));
}

int attn_gemm_act(const void* A, int64_t lda, int a_trans, const void* B, int64_t ldb, int b_trans,
                  int ab_dtype, void* C, int64_t ldc, int c_dtype, const float* bias, int M, int N, int K, int act,
                  void* aux, int64_t ldaux, int aux_dtype, void* stream) {
  clear_error();
  ATTN_REQUIRE(A && B && C, "attn_gemm_act: null pointer argument");
  ATTN_REQUIRE(M > 0 && N > 0 && K > 0, "attn_gemm_act: M, N, K must be positive");
  ATTN_REQUIRE(ab_dtype == ATTN_F32 || ab_dtype == ATTN_BF16 || ab_dtype == ATTN_TF32,
               "attn_gemm_act: bad operand dtype");
  ATTN_REQUIRE(c_dtype == ATTN_F32 || c_dtype == ATTN_BF16, "attn_gemm_act: bad output dtype");
  ATTN_REQUIRE(aux_dtype == ATTN_F32 || aux_dtype == ATTN_BF16, "attn_gemm_act: bad aux dtype");
  ATTN_REQUIRE(act == ATTN_ACT_NONE || act == ATTN_ACT_GELU || act == ATTN_ACT_GELU_BWD,
               "attn_gemm_act: unknown activation %d", act);
  ATTN_REQUIRE(act != ATTN_ACT_GELU_BWD || aux, "attn_gemm_act: ATTN_ACT_GELU_BWD needs the pre-activation aux");
  ATTN_REQUIRE(!aux || ldaux >= N, "attn_gemm_act: ldaux too small");
  ATTN_REQUIRE(!aux || (aux != C), "attn_gemm_act: aux and C must not alias");
  ATTN_REQUIRE(lda >= (a_trans ? M : K) && ldb >= (b_trans ? K : N) && ldc >= N,
               "attn_gemm_act: leading dimensions too small");
  if (act == ATTN_ACT_NONE) aux = nullptr;
  const int tf32 = ab_dtype == ATTN_TF32;
  if (ab_dtype != ATTN_F32 && tc_gemm_supported(M, N, K, lda, a_trans, ldb, b_trans, A, B, tf32) &&
      tc_gemm_act_ok(C, ldc, c_dtype, act, aux, ldaux, aux_dtype))
    return gemm_tc(A, lda, a_trans, B, ldb, b_trans, C, ldc, c_dtype, bias, M, N, K, 0, as_stream(stream), act,
                   aux, ldaux, aux_dtype, tf32);
  return gemm_simt(A, lda, a_trans, B, ldb, b_trans, tf32 ? ATTN_F32 : ab_dtype, C, ldc, c_dtype, bias, M, N, K,
                   0, as_stream(stream), act, aux, ldaux, aux_dtype);
}

size_t attn_colsum_workspace_size(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  return colsum_ws(M, N);
}

int attn_colsum(const void* X, int x_dtype, int64_t ldx, int M, int N, float* out, int accumulate,
                void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  ATTN_REQUIRE(X && out, "attn_colsum: null pointer argument");
  ATTN_REQUIRE(M > 0 && N > 0 && ldx >= N, "attn_colsum: bad shape");
  ATTN_REQUIRE(x_dtype == ATTN_F32 || x_dtype == ATTN_BF16, "attn_colsum: bad dtype");
  if (!workspace || workspace_bytes < colsum_ws(M, N)) {
    set_error("attn_colsum: workspace of %zu bytes required", colsum_ws(M, N));
    return ATTN_ERR_WORKSPACE;
  }
  return colsum(X, x_dtype, ldx, M, N, out, accumulate, workspace, as_stream(stream));
}

int attn_cast_colsum_f32(const float* X, int64_t ldx, int M, int N, void* Y, int64_t ldy, float* out,
                         int accumulate, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  ATTN_REQUIRE(X && Y && out, "attn_cast_colsum_f32: null pointer argument");
  ATTN_REQUIRE(M > 0 && N > 0 && ldx >= N && ldy >= N, "attn_cast_colsum_f32: bad shape");
  if (!workspace || workspace_bytes < colsum_ws(M, N)) {
    set_error("attn_cast_colsum_f32: workspace of %zu bytes required", colsum_ws(M, N));
    return ATTN_ERR_WORKSPACE;
  }
  return cast_colsum(X, ldx, M, N, Y, ldy, out, accumulate, workspace, as_stream(stream));
}

int attn_cast_rows_ones_bf16(const float* x, int64_t ldx, int M, int N, void* y, int64_t ldy,
                             void* stream) {
  clear_error();
  ATTN_REQUIRE(x && y, "attn_cast_rows_ones_bf16: null pointer argument");
  ATTN_REQUIRE(M > 0 && N > 0 && ldx >= N, "attn_cast_rows_ones_bf16: bad shape");
  ATTN_REQUIRE(ldy > N && ldy % 8 == 0, "attn_cast_rows_ones_bf16: ldy must exceed N and be a multiple of 8");
  ATTN_REQUIRE(aligned(y, 16), "attn_cast_rows_ones_bf16: y must be 16-byte aligned");
  return cast_rows_ones(x, ldx, M, N, y, ldy, as_stream(stream), sm_count());
}

int attn_layernorm(const float* x, int64_t ldx, const float* gamma, const float* beta, int M, int C,
                   float eps, void* y, int64_t ldy, int y_dtype, int ones_col, void* stream) {
  clear_error();
  ATTN_REQUIRE(x && gamma && beta && y, "attn_layernorm: null pointer argument");
  ATTN_REQUIRE(M > 0 && C > 0 && ldx >= C, "attn_layernorm: bad shape");
  ATTN_REQUIRE(y_dtype == ATTN_F32 || y_dtype == ATTN_BF16, "attn_layernorm: bad output dtype");
  ATTN_REQUIRE(ldy >= C + (ones_col ? 1 : 0), "attn_layernorm: ldy too small");
  ATTN_REQUIRE(eps > 0.f, "attn_layernorm: eps must be positive");
  ATTN_REQUIRE((const void*)x != (const void*)y, "attn_layernorm: x and y must not alias");
  return layernorm_rows(x, ldx, gamma, beta, M, C, eps, y, ldy, y_dtype, ones_col, as_stream(stream));
}

int attn_layernorm_bwd(const float* dy, const float* x, const float* gamma, int M, int C, float eps, float* dx,
                       int accumulate_dx, float* dgamma, float* dbeta, int accumulate_params, void* stream) {
  clear_error();
  ATTN_REQUIRE(dy && x && gamma && dx && dgamma && dbeta, "attn_layernorm_bwd: null pointer argument");
  ATTN_REQUIRE(M > 0 && C > 0, "attn_layernorm_bwd: bad shape");
  ATTN_REQUIRE(eps > 0.f, "attn_layernorm_bwd: eps must be positive");
  ATTN_REQUIRE((const void*)dx != (const void*)x && (const void*)dx != (const void*)dy,
               "attn_layernorm_bwd: dx must not alias x or dy");
  return layernorm_bwd_rows(dy, x, gamma, M, C, eps, dx, accumulate_dx, dgamma, dbeta, accumulate_params,
                            as_stream(stream), sm_count());
}

int attn_cast_f32_to_bf16(const float* x, void* y, int64_t n, void* stream) {
  clear_error();
  ATTN_REQUIRE(x && y && n > 0, "attn_cast_f32_to_bf16: bad argument");
  return cast_f32_bf16(x, y, n, as_stream(stream), sm_count());
}

int attn_split_heads(const float* qkv, float* q, float* k, float* v, int B, int T, int NH, int HD,
                     void* stream) {
  clear_error();
  ATTN_REQUIRE(qkv && q && k && v, "attn_split_heads: null pointer argument");
  ATTN_REQUIRE(B > 0 && T > 0 && NH > 0 && HD > 0, "attn_split_heads: sizes must be positive");
  return split_heads(qkv, q, k, v, B, T, NH, HD, as_stream(stream));
}

int attn_merge_heads(const float* ctx_heads, float* ctx, int B, int T, int NH, int HD, void* stream) {
  clear_error();
  ATTN_REQUIRE(ctx_heads && ctx, "attn_merge_heads: null pointer argument");
  ATTN_REQUIRE(B > 0 && T > 0 && NH > 0 && HD > 0, "attn_merge_heads: sizes must be positive");
  return merge_heads(ctx_heads, ctx, B, T, NH, HD, as_stream(stream));
}

}  // extern "C"
