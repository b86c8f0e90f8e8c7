// Fused causal / full attention backward for sm_100a (grxDNN). The reference
// has no attention at all (planned only: docs/designs/grxcp_roadmap.md:
// 864-865); this is the training-pass counterpart of attention.cu.
//
// With S = Q K^T, P = exp(scale S - LSE) (LSE saved by the forward), and
// Delta_q = sum_d dO[q, d] O[q, d]:
//   dV = P^T dO,   dP = dO V^T,   dS = P * (dP - Delta),
//   dK = scale dS^T Q,   dQ = scale dS K.
// Three launches, no atomics (bit-reproducible):
//   attn_bwd_delta_kernel   Delta, one warp per query row.
//   attn_bwd_kernel<kModeKV>  one CTA per (batch, head, 128-key block): K_j and
//       V_j stay in shared memory while the CTA walks the query blocks that see
//       them; dV_j and dK_j accumulate in TMEM.
//   attn_bwd_kernel<kModeQ>   one CTA per (batch, head, 128-query block): Q_i
//       and dO_i stay resident while it walks the key blocks; dQ_i accumulates
//       in TMEM. It recomputes S and dP instead of sharing dS with the KV
//       kernel through fp32 atomics.
// CTA: 320 threads. Warp 0 is the TMA producer (one thread): the resident pair
// once, then the streamed pair of each block through a 2-stage ring. Warp 1 is
// the MMA issuer (one thread): per block S = Q K^T and dP = dO V^T (K-major
// operands, 128 x 128 x 128 each), then dV += P^T dO and dK += dS^T Q (KV
// kernel) or dQ += dS K (Q kernel). Warps 2..9, two per TMEM lane quadrant
// (thread = query row; warp w takes columns [64 (w-2)/4, +64)), read S and dP
// from TMEM 32 columns at a time, form P and dS in fp32 and
// write them as bf16 into one 128 x 128 shared-memory tile in the same
// 128-byte-swizzled layout TMA gives a loaded tile (rows = queries). Read
// with a K-major descriptor that tile is the A operand for dQ (M = queries);
// read with an MN-major descriptor it is the A operand P^T / dS^T for dV / dK
// (M = keys). In the KV kernel the tile holds P first and dS second (dS waits
// in registers as packed bf16 while dV reads P).
// TMEM (512 columns): S [0,128), dP [128,256), dV or dQ [256,384), dK
// [384,512). All waits are bounded (ptx.cuh).
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "attention.cuh"
#include "profile.h"
#include "ptx.cuh"

namespace grx {

namespace {

constexpr int kD = 128;
constexpr int kB = 128;                   // queries or keys per block
constexpr int kTile = kB * kD * 2;        // 32 KiB bf16 tile (two 16 KiB swizzle halves)
constexpr int kHalf = 16384;
constexpr int kThreads = 320;
constexpr int kComputeWarps = 8;  // two per TMEM lane quadrant, one per 64-column half
constexpr int kModeKV = 0, kModeQ = 1;
// Resident pair (K,V or Q,dO), a 2-stage ring of streamed pairs, the P/dS tile.
constexpr int kSmem = 2 * kTile + 2 * 2 * kTile + kTile + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdParams {
  int batch, heads, seq_q, seq_k, n_qb, n_kb, causal;
  float scale, scale_log2;
  const float* lse;    // [batch, heads, seq_q] natural log
  const float* delta;  // [batch, heads, seq_q]
  void* out0;          // KV kernel: dK; Q kernel: dQ
  long long o0_sb, o0_sh, o0_ss;
  void* out1;          // KV kernel: dV
  long long o1_sb, o1_sh, o1_ss;
  int* err_word;
  unsigned long long timeout_ns;
};

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

// K-major operand: 128 rows x 128 bf16 as two 64-element swizzle halves; kk
// selects the 16-element k slice.
__device__ __forceinline__ uint64_t kmajor(uint32_t base, int kk) {
  return sw128_desc(base + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}
// The same tile read MN-major (its rows are the k index): kk selects 16 rows;
// the two 64-column halves are the two MN atoms, kHalf apart.
__device__ __forceinline__ uint64_t mnmajor(uint32_t base, int kk) {
  return sw128_desc(base + kk * 2048, kHalf, 1024);
}

// Byte offset of the 16-byte group holding columns [c, c + 8) of row r in a
// swizzled tile (c a multiple of 8).
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  return (uint32_t)((c >> 6) * kHalf + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Delta[q] = sum_d dO[q, d] O[q, d] in fp32, one warp per query row.
__global__ void attn_bwd_delta_kernel(int batch, int heads, int seq, const __nv_bfloat16* __restrict__ o,
                                      long long o_sb, long long o_sh, long long o_ss,
                                      const __nv_bfloat16* __restrict__ dout, long long d_sb, long long d_sh,
                                      long long d_ss, float* __restrict__ delta) {
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long rows = (long long)batch * heads * seq;
  if (row >= rows) return;
  const int s = (int)(row % seq);
  const long long bh = row / seq;
  const int h = (int)(bh % heads), b = (int)(bh / heads);
  const uint2 ov = *reinterpret_cast<const uint2*>(o + b * o_sb + h * o_sh + s * o_ss + lane * 4);
  const uint2 dv = *reinterpret_cast<const uint2*>(dout + b * d_sb + h * d_sh + s * d_ss + lane * 4);
  const __nv_bfloat162* op = reinterpret_cast<const __nv_bfloat162*>(&ov);
  const __nv_bfloat162* dp = reinterpret_cast<const __nv_bfloat162*>(&dv);
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float2 a = __bfloat1622float2(op[e]), c = __bfloat1622float2(dp[e]);
    acc = fmaf(a.x, c.x, acc);
    acc = fmaf(a.y, c.y, acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) delta[row] = acc;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const __grid_constant__ BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sRes = smem;              // KV: K, V.  Q: Q, dO.
  uint8_t* sRing = sRes + 2 * kTile;  // stage s: pair at s * 2 * kTile (KV: Q, dO.  Q: K, V)
  uint8_t* sPS = sRing + 4 * kTile;   // P / dS tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(sPS + kTile);
  uint64_t* res_full = bars;
  uint64_t* ring_full = bars + 1;   // [2]
  uint64_t* ring_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;      // S and dP in TMEM
  uint64_t* p_full = bars + 6;      // KV: P in smem, S/dP read (4 warps)
  uint64_t* ps_read = bars + 7;     // KV: dV has consumed P
  uint64_t* ds_full = bars + 8;     // dS in smem (4 warps); Q: also S/dP read
  uint64_t* ps_free = bars + 9;     // the MMA reading dS has completed
  uint64_t* acc_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_own = MODE == kModeKV ? p.n_kb : p.n_qb;
  const int bh = blockIdx.x / n_own;
  const int r_idx = blockIdx.x - bh * n_own;
  // KV: key block r (block 0 sees the most query blocks under a causal mask).
  // Q: query blocks from the last (longest causal row of key blocks) down.
  const int own = MODE == kModeKV ? r_idx : p.n_qb - 1 - r_idx;
  const int bi = bh / p.heads, hi = bh - bi * p.heads;
  const int it0 = (MODE == kModeKV && p.causal) ? own : 0;
  const int n_it = MODE == kModeKV ? p.n_qb - it0 : (p.causal ? min(own + 1, p.n_kb) : p.n_kb);

  if (threadIdx.x == 0) {
    mbar_init(res_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ring_full[s], 1);
      mbar_init(&ring_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, kComputeWarps);
    mbar_init(ps_read, 1);
    mbar_init(ds_full, kComputeWarps);
    mbar_init(ps_free, 1);
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmdO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  WaitCtx wc{p.err_word, abort_flag, p.timeout_ns};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const CUtensorMap* r0 = MODE == kModeKV ? &tmK : &tmQ;
      const CUtensorMap* r1 = MODE == kModeKV ? &tmV : &tmdO;
      const CUtensorMap* s0 = MODE == kModeKV ? &tmQ : &tmK;
      const CUtensorMap* s1 = MODE == kModeKV ? &tmdO : &tmV;
      mbar_arrive_expect_tx(res_full, 2 * kTile);
      for (int h = 0; h < 2; ++h) {
        tma_load_4d(sRes + h * kHalf, r0, res_full, h * 64, own * kB, hi, bi);
        tma_load_4d(sRes + kTile + h * kHalf, r1, res_full, h * 64, own * kB, hi, bi);
      }
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      for (int t = 0; t < n_it; ++t) {
        const int st = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!wait_bounded(&ring_empty[st], ph ^ 1u, wc, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        const int blk = it0 + t;
        uint8_t* dst = sRing + st * 2 * kTile;
        mbar_arrive_expect_tx(&ring_full[st], 2 * kTile);
        for (int h = 0; h < 2; ++h) {
          tma_load_4d(dst + h * kHalf, s0, &ring_full[st], h * 64, blk * kB, hi, bi);
          tma_load_4d(dst + kTile + h * kHalf, s1, &ring_full[st], h * 64, blk * kB, hi, bi);
        }
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      drain_wait(res_full, 0, p.timeout_ns, p.err_word);
      if (!ok)
        for (int s = 0; s < 2; ++s)
          if (armed & (1u << s)) drain_wait(&ring_full[s], (armed_par >> s) & 1u, p.timeout_ns, p.err_word);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc(1, 1, 1, 0, 0, 128, 128);   // S, dP: both K-major
      constexpr uint32_t idesc_kv = make_idesc(1, 1, 1, 1, 1, 128, 128);  // dV, dK: P^T / dS^T and dO / Q MN-major
      constexpr uint32_t idesc_q = make_idesc(1, 1, 1, 0, 1, 128, 128);   // dQ: dS K-major, K MN-major
      const uint32_t res = smem_u32(sRes), ring = smem_u32(sRing), ps = smem_u32(sPS);
      auto q_of = [&](int t) { return MODE == kModeKV ? ring + (t & 1) * 2 * kTile : res; };
      auto do_of = [&](int t) { return q_of(t) + kTile; };
      auto k_of = [&](int t) { return MODE == kModeKV ? res : ring + (t & 1) * 2 * kTile; };
      auto v_of = [&](int t) { return k_of(t) + kTile; };
      auto scores = [&](int t) {
        const uint32_t qa = q_of(t), ka = k_of(t), da = do_of(t), va = v_of(t);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_ss<0>(tmem, kmajor(qa, kk), kmajor(ka, kk), idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ss<0>(tmem + 128, kmajor(da, kk), kmajor(va, kk), idesc_s, kk > 0 ? 1u : 0u);
        mma_commit(s_full);
      };
      bool ok = wait_bounded(res_full, 0, wc, kErrTimeoutMma) && wait_bounded(&ring_full[0], 0, wc, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        scores(0);
      }
      for (int t = 0; t < n_it && ok; ++t) {
        const bool next = t + 1 < n_it;
        if (MODE == kModeKV) {
          if (!wait_bounded(p_full, t & 1, wc, kErrTimeoutMma)) break;
          tc_fence_after();
          const uint32_t da = do_of(t);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss<0>(tmem + 256, mnmajor(ps, kk), mnmajor(da, kk), idesc_kv, (t > 0 || kk > 0) ? 1u : 0u);
          mma_commit(ps_read);
          if (next) {
            if (!wait_bounded(&ring_full[(t + 1) & 1], ((t + 1) >> 1) & 1, wc, kErrTimeoutMma)) break;
            tc_fence_after();
            scores(t + 1);
          }
          if (!wait_bounded(ds_full, t & 1, wc, kErrTimeoutMma)) break;
          tc_fence_after();
          const uint32_t qa = q_of(t);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss<0>(tmem + 384, mnmajor(ps, kk), mnmajor(qa, kk), idesc_kv, (t > 0 || kk > 0) ? 1u : 0u);
        } else {
          if (!wait_bounded(ds_full, t & 1, wc, kErrTimeoutMma)) break;
          tc_fence_after();
          if (next) {
            if (!wait_bounded(&ring_full[(t + 1) & 1], ((t + 1) >> 1) & 1, wc, kErrTimeoutMma)) break;
            tc_fence_after();
            scores(t + 1);
          }
          const uint32_t ka = k_of(t);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss<0>(tmem + 256, kmajor(ps, kk), mnmajor(ka, kk), idesc_q, (t > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(ps_free);
        mma_commit(&ring_empty[t & 1]);
      }
      mma_commit(acc_done);
      // Every MMA this thread issued must complete before TMEM is released.
      mma_commit(drain);
      drain_wait(drain, 0, p.timeout_ns, p.err_word);
    }
  } else {
    // ------------------------------------------------------------ P / dS and the epilogue
    const int q = warp & 3;
    const int cb = ((warp - 2) >> 2) * 64;  // this warp's 64 of the 128 key (or head-dim) columns
    const int row = q * 32 + lane;
    const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t ps = smem_u32(sPS);
    const long long stat_base = (long long)bh * p.seq_q;
    bool ok = true;
    for (int t = 0; t < n_it && ok; ++t) {
      const int qblk = MODE == kModeKV ? it0 + t : own;
      const int kblk = MODE == kModeKV ? own : t;
      const int qabs = qblk * kB + row;
      const bool qvalid = qabs < p.seq_q;
      const float lse_l2 = qvalid ? p.lse[stat_base + qabs] * kLog2e : 0.f;
      const float dlt = qvalid ? p.delta[stat_base + qabs] : 0.f;
      if (!wait_bounded(s_full, t & 1, wc, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      // The P/dS tile still holds the previous block's dS until its MMA ends.
      if (t > 0 && !wait_bounded(ps_free, (t - 1) & 1, wc, kErrTimeoutEpilogue)) break;
      uint32_t ds_pk[MODE == kModeKV ? 32 : 1];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int col = cb + c * 32;
        uint32_t rs[32], rd[32];
        tmem_ld_32x32b_x32(t_row + col, rs);
        tmem_ld_32x32b_x32(t_row + 128 + col, rd);
        tmem_ld_wait();
        uint32_t pp[16], dd[16];
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          float pv[2], dv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int k = kblk * kB + col + jj + e;
            const bool valid = qvalid && k < p.seq_k && (!p.causal || k <= qabs);
            pv[e] = valid ? ex2_approx(fmaf(__uint_as_float(rs[jj + e]), p.scale_log2, -lse_l2)) : 0.f;
            dv[e] = pv[e] * (__uint_as_float(rd[jj + e]) - dlt);
          }
          pp[jj / 2] = pack_bf16(pv[0], pv[1]);
          dd[jj / 2] = pack_bf16(dv[0], dv[1]);
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (MODE == kModeKV) {
            st_shared_v4(ps + swz_off(row, col + g * 8), pp[4 * g], pp[4 * g + 1], pp[4 * g + 2], pp[4 * g + 3]);
#pragma unroll
            for (int e = 0; e < 4; ++e) ds_pk[c * 16 + 4 * g + e] = dd[4 * g + e];
          } else {
            st_shared_v4(ps + swz_off(row, col + g * 8), dd[4 * g], dd[4 * g + 1], dd[4 * g + 2], dd[4 * g + 3]);
          }
        }
      }
      tc_fence_before();
      fence_async_smem();
      __syncwarp();
      if (MODE == kModeKV) {
        if (lane == 0) mbar_arrive(p_full);
        // dS replaces P once dV has read it.
        if (!wait_bounded(ps_read, t & 1, wc, kErrTimeoutEpilogue)) break;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int g = 0; g < 4; ++g)
            st_shared_v4(ps + swz_off(row, cb + c * 32 + g * 8), ds_pk[c * 16 + 4 * g], ds_pk[c * 16 + 4 * g + 1],
                         ds_pk[c * 16 + 4 * g + 2], ds_pk[c * 16 + 4 * g + 3]);
        fence_async_smem();
        __syncwarp();
      }
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (ok && wait_bounded(acc_done, 0, wc, kErrTimeoutEpilogue) && !*abort_flag) {
      tc_fence_after();
      // KV: dK (scaled) from [384, 512) to out0, dV from [256, 384) to out1.
      // Q: dQ (scaled) from [256, 384) to out0.
      const int rabs = own * kB + row;
      const bool rvalid = rabs < (MODE == kModeKV ? p.seq_k : p.seq_q);
      for (int which = 0; which < (MODE == kModeKV ? 2 : 1); ++which) {
        const uint32_t col = MODE == kModeKV ? (which == 0 ? 384u : 256u) : 256u;
        const float mul = which == 0 ? p.scale : 1.f;
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(which == 0 ? p.out0 : p.out1) +
                             (which == 0 ? (long long)bi * p.o0_sb + (long long)hi * p.o0_sh + (long long)rabs * p.o0_ss
                                         : (long long)bi * p.o1_sb + (long long)hi * p.o1_sh + (long long)rabs * p.o1_ss);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + col + cb + c * 32, v);
          tmem_ld_wait();
          if (rvalid) {
            uint4* dst = reinterpret_cast<uint4*>(out + cb + c * 32);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                w[e] = pack_bf16(__uint_as_float(v[8 * g + 2 * e]) * mul, __uint_as_float(v[8 * g + 2 * e + 1]) * mul);
              dst[g] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
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
// A batch or head stride of 0 (broadcast) is replaced by the dense stride the
// map needs for a dimension of extent 1.
bool make_map(CUtensorMap* m, const void* base, int batch, int heads, int seq, long long sb, long long sh,
              long long ss) {
  if (batch == 1) sb = (long long)heads * sh;
  if (heads == 1) sh = (long long)seq * ss;
  if (sb == 0) sb = 8;
  if (sh == 0) sh = 8;
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

template <int MODE>
cudaError_t launch_mode(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& md,
                        const BwdParams& p, cudaStream_t s) {
  auto kfn = attn_bwd_kernel<MODE>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] { attr = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem); });
  if (attr != cudaSuccess) return attr;
  const long long grid = (long long)(MODE == kModeKV ? p.n_kb : p.n_qb) * p.batch * p.heads;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  ProfLaunch prof(MODE == kModeKV ? "attn_bwd_kernel<dKdV>" : "attn_bwd_kernel<dQ>", dim3((unsigned)grid),
                  dim3(kThreads), kSmem, s);
  kfn<<<(unsigned)grid, kThreads, kSmem, s>>>(mq, mk, mv, md, p);
  return cudaGetLastError();
}

}  // namespace

size_t attention_bwd_workspace_bytes(const AttnBwdArgs& a) {
  return (size_t)a.batch * a.heads * a.seq_q * sizeof(float);
}

cudaError_t launch_attention_bwd(const AttnBwdArgs& a, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (!ws || ws_bytes < attention_bwd_workspace_bytes(a)) return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mv, md;
  if (!make_map(&mq, a.q, a.batch, a.heads, a.seq_q, a.q_sb, a.q_sh, a.q_ss) ||
      !make_map(&mk, a.k, a.batch, a.heads, a.seq_k, a.k_sb, a.k_sh, a.k_ss) ||
      !make_map(&mv, a.v, a.batch, a.heads, a.seq_k, a.v_sb, a.v_sh, a.v_ss) ||
      !make_map(&md, a.dout, a.batch, a.heads, a.seq_q, a.do_sb, a.do_sh, a.do_ss))
    return cudaErrorNotSupported;
  const void* outs[3] = {a.dq, a.dk, a.dv};
  const long long oss[3] = {a.dq_ss, a.dk_ss, a.dv_ss};
  for (int i = 0; i < 3; ++i)
    if ((reinterpret_cast<uintptr_t>(outs[i]) & 15u) || (oss[i] * 2) % 16) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(a.o) & 7u) || (reinterpret_cast<uintptr_t>(a.dout) & 7u)) return cudaErrorNotSupported;
  float* delta = static_cast<float*>(ws);
  {
    const long long rows = (long long)a.batch * a.heads * a.seq_q;
    const long long blocks = (rows + 7) / 8;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    ProfLaunch prof("attn_bwd_delta_kernel", dim3((unsigned)blocks), dim3(256), 0, s);
    attn_bwd_delta_kernel<<<(unsigned)blocks, 256, 0, s>>>(
        a.batch, a.heads, a.seq_q, static_cast<const __nv_bfloat16*>(a.o), a.o_sb, a.o_sh, a.o_ss,
        static_cast<const __nv_bfloat16*>(a.dout), a.do_sb, a.do_sh, a.do_ss, delta);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  BwdParams p{};
  p.batch = a.batch;
  p.heads = a.heads;
  p.seq_q = a.seq_q;
  p.seq_k = a.seq_k;
  p.n_qb = (a.seq_q + kB - 1) / kB;
  p.n_kb = (a.seq_k + kB - 1) / kB;
  p.causal = a.causal;
  p.scale = a.scale;
  p.scale_log2 = a.scale * kLog2e;
  p.lse = a.lse;
  p.delta = delta;
  p.err_word = a.err_word;
  p.timeout_ns = a.timeout_ns;
  p.out0 = a.dk;
  p.o0_sb = a.dk_sb; p.o0_sh = a.dk_sh; p.o0_ss = a.dk_ss;
  p.out1 = a.dv;
  p.o1_sb = a.dv_sb; p.o1_sh = a.dv_sh; p.o1_ss = a.dv_ss;
  cudaError_t e = launch_mode<kModeKV>(mq, mk, mv, md, p, s);
  if (e != cudaSuccess) return e;
  p.out0 = a.dq;
  p.o0_sb = a.dq_sb; p.o0_sh = a.dq_sh; p.o0_ss = a.dq_ss;
  p.out1 = nullptr;
  return launch_mode<kModeQ>(mq, mk, mv, md, p, s);
}

}  // namespace grx
