// tcgen05 tensor-core causal attention forward for head_dim 64, bf16 operands, fp32 accumulation.
//
// Replaces fused_attention_forward_kernel (core/mha_kernels.py:404-521): one CTA per
// (b, h, 128-row query tile), two CTAs per SM.  Per 128-key K/V block:
//   S = Q K^T           tcgen05.mma, A = Q and B = K from shared memory (TMA, 128B swizzle),
//                       fp32 accumulator in TMEM columns [0,128)
//   softmax             4 warps, one query row per thread (tcgen05.ld of its TMEM lane): causal
//                       mask on the diagonal block, row max, 2^(s*scale*log2e - m), row sum; P is
//                       packed to bf16 and written back over S in TMEM columns [0,64)
//   O += P V            tcgen05.mma with A = P read from TMEM, B = V (MN-major) from shared
//                       memory, fp32 accumulator in TMEM columns [128,192)
// The running max is only moved (and O rescaled in TMEM) when it grows by more than 2^8, so
// rescaling is rare.  The row's log-sum-exp is written instead of the T x T probabilities.
//
// Every mbarrier wait is bounded (tc_common.cuh): a wait that gives up sets the library's device
// error word and the kernel skips its remaining work instead of hanging.
#include "attn_tc_common.cuh"

#include <math.h>

namespace attn {

// ==========================================================================================
// forward
// ==========================================================================================
constexpr int FA_THREADS = 192;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 softmax/epilogue
constexpr int FA_STAGES = 2;
constexpr uint32_t FA_TMEM_COLS = 256;  // S/P [0,128), O [128,192)
constexpr int FA_SMEM = AT_TILE_BYTES * (1 + 2 * FA_STAGES) + 1024 + 256;

struct FwdMaps {
  TileMap q, k, v;
};

struct FwdParams {
  int NH, T, nq;
  float scale_log2;
  __nv_bfloat16* o;
  int64_t o_sb, o_st, o_sh;
  float* lse;
  int* err;
};

__global__ void __launch_bounds__(FA_THREADS, 2)
attn_fwd_tc_kernel(const __grid_constant__ FwdMaps maps, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + AT_TILE_BYTES;                      // [FA_STAGES]
  uint8_t* sV = sK + FA_STAGES * AT_TILE_BYTES;            // [FA_STAGES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + FA_STAGES * AT_TILE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + FA_STAGES;
  uint64_t* kv_empty = v_full + FA_STAGES;
  uint64_t* s_full = kv_empty + FA_STAGES;
  uint64_t* p_ready = s_full + 1;
  uint64_t* pv_done = p_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x / p.nq;
  const int qt = p.nq - 1 - (int)(blockIdx.x % p.nq);  // longest causal rows first within a head
  const int b = bh / p.NH, h = bh % p.NH;
  const int n_kv = qt + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < FA_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_ready, 128);
    mbar_init(pv_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, FA_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tP = tmem, tO = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&maps.q.map);
      tma_prefetch_desc(&maps.k.map);
      tma_prefetch_desc(&maps.v.map);
      mbar_arrive_expect_tx(q_full, AT_TILE_BYTES);
      load_tile(sQ, maps.q, q_full, b, h, qt * AT_TILE);
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % FA_STAGES;
        const uint32_t ph = (j / FA_STAGES) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, p.err, 201)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[st], AT_TILE_BYTES);
        load_tile(sK + st * AT_TILE_BYTES, maps.k, &k_full[st], b, h, j * AT_TILE);
        mbar_arrive_expect_tx(&v_full[st], AT_TILE_BYTES);
        load_tile(sV + st * AT_TILE_BYTES, maps.v, &v_full[st], b, h, j * AT_TILE);
      }
      // tail: every stage released by the MMA thread before the CTA may exit
      for (int j = n_kv; j < n_kv + FA_STAGES && ok; ++j)
        ok = mbar_wait(&kv_empty[j % FA_STAGES], ((j / FA_STAGES) & 1) ^ 1, p.err, 202);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);  // Q K-major, K K-major
      const uint32_t idesc_o = idesc_bf16_f32(128, 64, 0, 1);   // P from TMEM, V MN-major
      bool ok = mbar_wait(q_full, 0, p.err, 203);
      const uint32_t q_addr = smem_u32(sQ);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % FA_STAGES;
        const uint32_t ph = (j / FA_STAGES) & 1;
        if (!mbar_wait(&k_full[st], ph, p.err, 204)) break;
        if (j > 0 && !mbar_wait(pv_done, (j - 1) & 1, p.err, 205)) break;  // P_{j-1} consumed
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * AT_TILE_BYTES);
#pragma unroll
        for (int k = 0; k < AT_D / 16; ++k)
          umma_ss(tS, smem_desc_sw128(q_addr + k * 32, 16, 1024), smem_desc_sw128(k_addr + k * 32, 16, 1024),
                  idesc_s, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        if (!mbar_wait(p_ready, j & 1, p.err, 206)) break;
        if (!mbar_wait(&v_full[st], ph, p.err, 207)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * AT_TILE_BYTES);
#pragma unroll
        for (int k = 0; k < AT_TILE / 16; ++k)
          umma_ts(tO, tP + k * 8, smem_desc_sw128(v_addr + k * 2048, 8192, 1024), idesc_o,
                  (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(pv_done);
        umma_commit(&kv_empty[st]);
      }
    }
  } else {
    // ---------------- softmax warpgroup: one query row per thread ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int grow = qt * AT_TILE + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, p.err, 208));
      if (!ok) break;
      tc_fence_after();
      const bool diag = (j == qt);
      // pass 1: row max of the scaled scores (log2 domain)
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + lane_off + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float s = __uint_as_float(r[i]);
          const bool masked = diag && (c * 32 + i > row);
          mx = masked ? mx : fmaxf(mx, s);
        }
      }
      const float m_cand = mx * sl2;
      // move the max (and rescale O) only when it grows by more than 8 in log2 units
      const bool grow_m = (j == 0) || (m_cand > m + 8.0f);
      if (j > 0 && __any_sync(0xffffffffu, grow_m)) {
        const float alpha = grow_m ? ex2_approx(m - m_cand) : 1.f;
        // O holds exactly PV_0..PV_{j-1}: S_j was issued only after PV_{j-1} completed
        uint32_t o0[32], o1[32];
        tmem_ld32(tO + lane_off, o0);
        tmem_ld32(tO + lane_off + 32, o1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          o0[i] = __float_as_uint(__uint_as_float(o0[i]) * alpha);
          o1[i] = __float_as_uint(__uint_as_float(o1[i]) * alpha);
        }
        uint32_t w[16];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const uint32_t* src = q4 < 2 ? o0 + 16 * q4 : o1 + 16 * (q4 - 2);
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = src[i];
          tmem_st16(tO + lane_off + 16 * q4, w);
        }
        l *= alpha;
      }
      if (grow_m) m = m_cand;
      // pass 2: probabilities, row sum, P (bf16) over the first 64 columns of S
      float sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + lane_off + c * 32, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const bool m0 = diag && (c * 32 + i > row);
          const bool m1 = diag && (c * 32 + i + 1 > row);
          const float p0 = m0 ? 0.f : ex2_approx(fmaf(__uint_as_float(r[i]), sl2, -m));
          const float p1 = m1 ? 0.f : ex2_approx(fmaf(__uint_as_float(r[i + 1]), sl2, -m));
          sum += p0 + p1;
          pk[i / 2] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tP + lane_off + c * 16, pk);
      }
      tmem_wait_st();
      l += sum;
      tc_fence_before();
      mbar_arrive(p_ready);
    }
    // epilogue: O / l -> bf16 rows, lse = (m + log2 l) * ln 2
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (n_kv - 1) & 1, p.err, 209));
    if (ok) {
      tc_fence_after();
      uint32_t o0[32], o1[32];
      tmem_ld32(tO + lane_off, o0);
      tmem_ld32(tO + lane_off + 32, o1);
      tmem_wait_ld();
      if (grow < p.T) {
        const float inv = 1.f / l;
        __nv_bfloat16* dst = p.o + (int64_t)b * p.o_sb + (int64_t)grow * p.o_st + (int64_t)h * p.o_sh;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* src = c < 4 ? o0 + 8 * c : o1 + 8 * (c - 4);
          uint4 u;
          u.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
          u.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
          u.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
          u.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
          reinterpret_cast<uint4*>(dst)[c] = u;
        }
        p.lse[(int64_t)bh * p.T + grow] = (m + __log2f(l)) * LN2;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, FA_TMEM_COLS);
  }
}

// ==========================================================================================
// host side
// ==========================================================================================
bool tc_fwd_supported(int D, int dtype) { return D == AT_D && dtype == ATTN_BF16; }

int attn_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH, int T,
                int D, const int64_t* s, float scale, cudaStream_t stream) {
  (void)D;
  if (!head_strides_ok(s[0], s[1], s[2]) || !head_strides_ok(s[3], s[4], s[5]) || !aligned(q, 16) || !aligned(k, 16) ||
      !aligned(v, 16) || !aligned(o, 16)) {
    set_error("attn_fwd: the tensor-core path needs 16-byte aligned bf16 tensors with strides that are "
              "multiples of 8 elements");
    return ATTN_ERR_ARG;
  }
  FwdMaps maps;
  if (!make_head_map(&maps.q, q, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.k, k, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.v, v, B, NH, T, s[0], s[1], s[2]))
    return ATTN_ERR_CUDA;
  FwdParams p;
  p.NH = NH;
  p.T = T;
  p.nq = (T + AT_TILE - 1) / AT_TILE;
  p.scale_log2 = scale * LOG2E;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.o_sb = s[3];
  p.o_st = s[4];
  p.o_sh = s[5];
  p.lse = lse;
  p.err = dev_error_ptr();
  if (!p.err) return ATTN_ERR_CUDA;
  static bool attr = false;
  if (!attr) {
    ATTN_CUDA_TRY(cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM));
    attr = true;
  }
  const int64_t grid = (int64_t)B * NH * p.nq;
  attn_fwd_tc_kernel<<<(unsigned)grid, FA_THREADS, FA_SMEM, stream>>>(maps, p);
  count_launch();
  return check_launch("attn_fwd_tc_kernel");
}

}  // namespace attn
