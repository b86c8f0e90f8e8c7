// Fused scaled-dot-product attention forward for sm_100a (grxDNN; the
// reference plans "fused attention" at docs/designs/grxcp_roadmap.md:864-865
// and implements none).
//
// One CTA per (batch, head, 128-query tile); causal grids launch the longest
// tiles first. 192 threads:
//   warp 0      TMA producer: Q tile once, then K and V tiles (128 keys x 128
//               dims, bf16, 128-byte swizzle) through a 2-stage ring.
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM
//               S buffers, then O += P_{j-1} V_{j-1} into the TMEM O
//               accumulator, so the tensor core computes block j+1's scores
//               while the softmax warps work on block j.
//   warps 2..5  softmax (thread = query row): read S_j from TMEM, mask,
//               online max/sum in the exp2 domain with the softmax scale
//               folded in, write P_j (bf16) into swizzled smem for the PV MMA;
//               rescale O in TMEM only when the running max grows by more than
//               2^8 (otherwise p <= 256 stays exact enough in fp32); at the
//               end normalise O, store bf16 O and the fp32 natural-log LSE.
// All waits are bounded (ptx.cuh).
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "attention.cuh"
#include "ptx.cuh"

namespace grx {

namespace {

constexpr int kD = 128;                   // head dim
constexpr int kBQ = 128;                  // queries per CTA
constexpr int kBK = 128;                  // keys per block
constexpr int kTileBytes = 128 * kD * 2;  // one 128 x 128 bf16 tile = 32 KiB (two 16 KiB swizzle halves)
constexpr int kHalf = 16384;
constexpr int kKvStages = 2;
constexpr int kThreads = 192;
constexpr int kSmem = kTileBytes /*Q*/ + kTileBytes /*P*/ + kKvStages * 2 * kTileBytes + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct AttnParams {
  int batch, heads, seq_q, seq_k, n_qt, n_kb, causal;
  float scale_log2;
  void* o;
  long long o_sb, o_sh, o_ss;
  float* lse;
  int* err_word;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __noinline__ void drain_wait(uint64_t* bar, uint32_t parity, uint64_t timeout_ns, int* err) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      if (err) atomicCAS(err, 0, kErrTimeoutDrain);
      return;
    }
  }
}

// K-major operand descriptor for a 128-row x 128-element (bf16) tile stored as
// two 64-element swizzle halves; kk selects the 16-element k slice.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return sw128_desc(base + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sP = sQ + kTileBytes;
  uint8_t* sKV = sP + kTileBytes;  // stage s: K at s*2T, V at s*2T + T
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kKvStages * 2 * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + kKvStages;
  uint64_t* kv_empty = v_full + kKvStages;
  uint64_t* s_full = kv_empty + kKvStages;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh_count = p.batch * p.heads;
  const int qt = p.causal ? (p.n_qt - 1 - (int)(blockIdx.x / bh_count)) : (int)(blockIdx.x / bh_count);
  const int bh = blockIdx.x % bh_count;
  const int bi = bh / p.heads, hi = bh % p.heads;
  const int nblk = p.causal ? min(qt + 1, p.n_kb) : p.n_kb;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S0 at +0, S1 at +128, O at +256
  WaitCtx wc{p.err_word, abort_flag, p.timeout_ns};

  if (warp == 0) {
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_4d(sQ, &tmQ, q_full, 0, qt * kBQ, hi, bi);
      tma_load_4d(sQ + kHalf, &tmQ, q_full, 64, qt * kBQ, hi, bi);
      for (int j = 0; j < nblk; ++j) {
        const int st = j % kKvStages;
        const uint32_t ph = (j / kKvStages) & 1;
        if (!wait_bounded(&kv_empty[st], ph ^ 1u, wc, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* sk = sKV + st * 2 * kTileBytes;
        uint8_t* sv = sk + kTileBytes;
        mbar_arrive_expect_tx(&k_full[st], kTileBytes);
        tma_load_4d(sk, &tmK, &k_full[st], 0, j * kBK, hi, bi);
        tma_load_4d(sk + kHalf, &tmK, &k_full[st], 64, j * kBK, hi, bi);
        mbar_arrive_expect_tx(&v_full[st], kTileBytes);
        tma_load_4d(sv, &tmV, &v_full[st], 0, j * kBK, hi, bi);
        tma_load_4d(sv + kHalf, &tmV, &v_full[st], 64, j * kBK, hi, bi);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      drain_wait(q_full, 0, p.timeout_ns, p.err_word);
      if (!ok) {
        for (int s = 0; s < kKvStages; ++s)
          if (armed & (1u << s)) {
            drain_wait(&k_full[s], (armed_par >> s) & 1u, p.timeout_ns, p.err_word);
            drain_wait(&v_full[s], (armed_par >> s) & 1u, p.timeout_ns, p.err_word);
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S = Q K^T: bf16 x bf16 -> f32, both K-major, M = N = 128.
      constexpr uint32_t idesc_s = make_idesc(1, 1, 1, 0, 0, 128, 128);
      // O += P V: P K-major (keys contiguous), V MN-major (dims contiguous).
      constexpr uint32_t idesc_o = make_idesc(1, 1, 1, 0, 1, 128, 128);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      bool ok = wait_bounded(q_full, 0, wc, kErrTimeoutMma);
      tc_fence_after();
      for (int j = 0; j <= nblk && ok; ++j) {
        if (j < nblk) {
          const int st = j % kKvStages;
          if (!wait_bounded(&k_full[st], (j / kKvStages) & 1, wc, kErrTimeoutMma)) break;
          if (!wait_bounded(&s_free[j & 1], ((j >> 1) & 1) ^ 1u, wc, kErrTimeoutMma)) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sKV + st * 2 * kTileBytes);
          const uint32_t d = tmem + (j & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss<0>(d, kmajor_desc(q_addr, kk), kmajor_desc(k_addr, kk), idesc_s, kk > 0 ? 1u : 0u);
          mma_commit(&s_full[j & 1]);
        }
        if (j > 0) {
          const int jp = j - 1;
          const int st = jp % kKvStages;
          if (!wait_bounded(&v_full[st], (jp / kKvStages) & 1, wc, kErrTimeoutMma)) break;
          if (!wait_bounded(p_full, jp & 1, wc, kErrTimeoutMma)) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sKV + st * 2 * kTileBytes + kTileBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss<0>(tmem + 256, kmajor_desc(p_addr, kk), sw128_desc(v_addr + kk * 2048, kHalf, 1024), idesc_o,
                      (jp > 0 || kk > 0) ? 1u : 0u);
          mma_commit(o_done);
          mma_commit(&kv_empty[st]);
        }
      }
      mma_commit(drain);
      drain_wait(drain, 0, p.timeout_ns, p.err_word);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const int qi = qt * kBQ + r;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    uint8_t* prow = sP + r * 128;
    for (int j = 0; j < nblk; ++j) {
      if (!wait_bounded(&s_full[j & 1], (j >> 1) & 1, wc, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tmem + lane_base + (j & 1) * 128 + c * 32, u);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(u[e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[j & 1]);

      const int key0 = j * kBK;
      const bool need_mask = (key0 + kBK > p.seq_k) || (p.causal && key0 + kBK - 1 > qt * kBQ);
      float mb = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        float v = s[c] * p.scale_log2;
        if (need_mask) {
          const int key = key0 + c;
          if (key >= p.seq_k || (p.causal && key > qi)) v = -INFINITY;
        }
        s[c] = v;
        mb = fmaxf(mb, v);
      }
      const float m_new = fmaxf(m_run, mb);
      const bool rescale = (j == 0) || (m_new > m_run + kRescaleThreshold);
      float m_use = rescale ? m_new : m_run;
      if (m_use == -INFINITY) m_use = 0.f;
      const float alpha = (rescale && j > 0) ? exp2f(m_run - m_use) : 1.f;
      float rs = 0.f;
      uint32_t packed[64];
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        const float p0 = exp2f(s[c] - m_use);
        const float p1 = exp2f(s[c + 1] - m_use);
        rs += p0 + p1;
        __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
        packed[c >> 1] = *reinterpret_cast<uint32_t*>(&h);
      }
      l_run = l_run * alpha + rs;
      m_run = m_use;

      if (j > 0) {
        // PV of the previous block must be done: it reads sP and writes O.
        if (!wait_bounded(o_done, (j - 1) & 1, wc, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t u[32];
            const uint32_t ta = tmem + lane_base + 256 + c * 32;
            tmem_ld_32x32b_x32(ta, u);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
            tmem_st_32x32b_x32(ta, u);
          }
          tmem_st_wait();
        }
      }
      // P row -> swizzled K-major smem (two 64-key halves, 16-byte chunks).
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        const int half = ch >> 3, c16 = ch & 7;
        uint4 val = make_uint4(packed[ch * 4], packed[ch * 4 + 1], packed[ch * 4 + 2], packed[ch * 4 + 3]);
        *reinterpret_cast<uint4*>(prow + half * kHalf + ((c16 ^ (r & 7)) << 4)) = val;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && wait_bounded(o_done, (nblk - 1) & 1, wc, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.o) + (long long)bi * p.o_sb + (long long)hi * p.o_sh +
                            (long long)qi * p.o_ss;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tmem + lane_base + 256 + c * 32, u);
        tmem_ld_wait();
        if (qi < p.seq_q) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(u[e + 2 * t]) * inv_l,
                                                       __uint_as_float(u[e + 2 * t + 1]) * inv_l);
              wp[t] = *reinterpret_cast<uint32_t*>(&h);
            }
            *reinterpret_cast<uint4*>(orow + c * 32 + e) = w;
          }
        }
      }
      if (p.lse && qi < p.seq_q)
        p.lse[((long long)bi * p.heads + hi) * p.seq_q + qi] = (m_run + log2f(l_run)) * kLn2;
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// [batch, heads, seq, 128] bf16 -> 4-D map {128, seq, heads, batch}, box {64, 128, 1, 1}.
bool make_bhsd_map(CUtensorMap* m, const void* base, int batch, int heads, int seq, long long sb, long long sh,
                   long long ss) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (ss * 2) % 16 || (sh * 2) % 16 || (sb * 2) % 16) return false;
  if (ss <= 0 || sh <= 0 || sb <= 0) return false;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)seq, (cuuint64_t)heads, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)(ss * 2), (cuuint64_t)(sh * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_attention_fwd(const AttnArgs& a, int num_sms, cudaStream_t s) {
  (void)num_sms;
  CUtensorMap mq, mk, mv;
  // A batch or head stride of 0 (broadcast) cannot be expressed: refuse.
  const long long q_sb = a.batch > 1 ? a.q_sb : (long long)a.heads * a.q_sh;
  const long long k_sb = a.batch > 1 ? a.k_sb : (long long)a.heads * a.k_sh;
  const long long v_sb = a.batch > 1 ? a.v_sb : (long long)a.heads * a.v_sh;
  const long long q_sh = a.heads > 1 ? a.q_sh : (long long)a.seq_q * a.q_ss;
  const long long k_sh = a.heads > 1 ? a.k_sh : (long long)a.seq_k * a.k_ss;
  const long long v_sh = a.heads > 1 ? a.v_sh : (long long)a.seq_k * a.v_ss;
  if (!make_bhsd_map(&mq, a.q, a.batch, a.heads, a.seq_q, q_sb ? q_sb : 8, q_sh ? q_sh : 8, a.q_ss) ||
      !make_bhsd_map(&mk, a.k, a.batch, a.heads, a.seq_k, k_sb ? k_sb : 8, k_sh ? k_sh : 8, a.k_ss) ||
      !make_bhsd_map(&mv, a.v, a.batch, a.heads, a.seq_k, v_sb ? v_sb : 8, v_sh ? v_sh : 8, a.v_ss))
    return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(a.o) & 15u) || (a.o_ss * 2) % 16) return cudaErrorNotSupported;
  AttnParams p{};
  p.batch = a.batch;
  p.heads = a.heads;
  p.seq_q = a.seq_q;
  p.seq_k = a.seq_k;
  p.n_qt = (a.seq_q + kBQ - 1) / kBQ;
  p.n_kb = (a.seq_k + kBK - 1) / kBK;
  p.causal = a.causal;
  p.scale_log2 = a.scale * kLog2e;
  p.o = a.o;
  p.o_sb = a.o_sb;
  p.o_sh = a.o_sh;
  p.o_ss = a.o_ss;
  p.lse = a.lse;
  p.err_word = a.err_word;
  p.timeout_ns = a.timeout_ns;
  const long long grid = (long long)p.n_qt * a.batch * a.heads;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (attr != cudaSuccess) return attr;
  attn_fwd_kernel<<<(unsigned)grid, kThreads, kSmem, s>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

}  // namespace grx
