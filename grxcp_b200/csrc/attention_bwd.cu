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
// once, then the streamed pair of each block half by half through a 4-stage
// ring of half-blocks (64 rows of both streamed tensors, 32 KiB): a stage is
// released as soon as that half's gradient MMAs are done, so the loads of the
// next block overlap a whole block of work (with whole-block stages of the same
// 128 KiB the MMA issuer waited ~2000 cycles per block for its next tile). Warp 1 is
// the MMA issuer (one thread). Warps 2..9 (two per TMEM lane quadrant) form P
// and dS. Each streamed block is worked in two halves of 64 (queries for the
// KV kernel, keys for the Q kernel) that ping-pong: while the compute warps
// turn half h's scores into P / dS, the tensor pipe runs the other half.
//   KV kernel, TMEM lanes = the CTA's 128 keys: S^T = K Q_h^T and
//       dP^T = V dO_h^T (N = 64); P^T and dS^T are written back as packed
//       bf16 over those columns and feed dV += P^T dO_h and dK += dS^T Q_h as
//       TS-MMAs (A from TMEM, B the streamed tile read MN-major).
//   Q kernel, TMEM lanes = the CTA's 128 queries: S = Q K_h^T, dP = dO V_h^T;
//       dS written back feeds dQ += dS K_h.
// The next block's scores for half h are issued right after half h's
// gradient MMAs (MMAs from one thread execute in order, so they land after
// those MMAs have read P / dS). Each compute warp packs its 32 columns into
// the first 16 of its own 32, so no warp writes columns another still reads.
// TMEM: dV or dQ [0,128), dK [128,256); half h scores at s_base + 128 h and
// its dP 64 columns further (s_base 256 for KV, 128 for Q). All waits are
// bounded (ptx.cuh).
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "attention.cuh"
#include "exp2_poly.cuh"
#include "profile.h"
#include "ptx.cuh"


namespace grx {

namespace {

constexpr int kD = 128;
constexpr int kB = 128;                   // queries or keys per block
constexpr int kTile = kB * kD * 2;        // 32 KiB bf16 tile (two 16 KiB swizzle halves)
constexpr int kHalf = 16384;
constexpr int kHS = 32768;                // half-block stage: 64 rows of each streamed tensor
constexpr int kRing = 4;                  // half-block stages
constexpr int kThreads = 320;
constexpr int kComputeWarps = 8;  // two per TMEM lane quadrant, one per 64-column half
constexpr int kModeKV = 0, kModeQ = 1;
// Resident pair (K,V or Q,dO) and the ring of streamed half-blocks.
constexpr int kSmem = 2 * kTile + kRing * kHS + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;
// Share of exponentials moved to the FMA pipe (every n-th pair; 0 = none). Measured at config 4:
// none 4.66 ms, 1/8 4.80, 1/4 4.93, 1/2 5.11 -- this stage is FMA-issue bound, not SFU bound.
constexpr int kPolyEveryBwd = 0;

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
// A half-block stage holds, per streamed tensor, 64 rows x 128 bf16 as two
// 64-element swizzle halves of 8 KiB. K-major read (rows = N of the scores):
__device__ __forceinline__ uint64_t kmajor_h(uint32_t base, int kk) {
  return sw128_desc(base + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
}
// The same 64 rows read MN-major (rows = the k index): kk selects 16 rows; the
// two 64-column halves are the two MN atoms, 8 KiB apart.
__device__ __forceinline__ uint64_t mnmajor_h(uint32_t base, int kk) {
  return sw128_desc(base + kk * 2048, 8192, 1024);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Delta[q] = sum_d dO[q, d] O[q, d] in fp32: 16 lanes per query row, one
// 16-byte load of O and of dO per lane, two rows per warp.
__global__ void attn_bwd_delta_kernel(int batch, int heads, int seq, const __nv_bfloat16* __restrict__ o,
                                      long long o_sb, long long o_sh, long long o_ss,
                                      const __nv_bfloat16* __restrict__ dout, long long d_sb, long long d_sh,
                                      long long d_ss, float* __restrict__ delta) {
  const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int part = threadIdx.x & 15;
  const long long rows = (long long)batch * heads * seq;
  const bool live = row < rows;
  float acc = 0.f;
  if (live) {
    const int s = (int)(row % seq);
    const long long bh = row / seq;
    const int h = (int)(bh % heads), b = (int)(bh / heads);
    const uint4 ov = __ldcs(reinterpret_cast<const uint4*>(o + b * o_sb + h * o_sh + s * o_ss) + part);
    const uint4 dv = __ldcs(reinterpret_cast<const uint4*>(dout + b * d_sb + h * d_sh + s * d_ss) + part);
    const __nv_bfloat162* op = reinterpret_cast<const __nv_bfloat162*>(&ov);
    const __nv_bfloat162* dp = reinterpret_cast<const __nv_bfloat162*>(&dv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = __bfloat1622float2(op[e]), c = __bfloat1622float2(dp[e]);
      acc = fmaf(a.x, c.x, acc);
      acc = fmaf(a.y, c.y, acc);
    }
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (live && part == 0) delta[row] = acc;
}

// Packed fp32 pairs (sm_100 executes f32x2 FMA / ADD / MUL as one instruction).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// TMEM column of the k-th 16-element slice of a half-block operand written by
// the compute warps: warp sub s of a quadrant packs its 32 columns (16 bf16
// pairs) at offset 32 s, so slices 0,1 sit at 0, 8 and slices 2,3 at 32, 40.
__device__ __forceinline__ uint32_t half_col(int kk) { return (uint32_t)((kk >> 1) * 32 + (kk & 1) * 8); }

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                    const __grid_constant__ BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sRes = smem;               // KV: K, V.  Q: Q, dO.
  // stage u % kRing of half-block u = 2 t + h: rows [64 h, 64 h + 64) of the
  // streamed pair (KV: Q, dO.  Q: K, V), first tensor at 0, second at 16 KiB.
  uint8_t* sRing = sRes + 2 * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + kRing * kHS);
  uint64_t* res_full = bars;
  uint64_t* ring_full = bars + 1;              // [kRing]
  uint64_t* ring_empty = bars + 1 + kRing;     // [kRing]
  uint64_t* s_full = bars + 1 + 2 * kRing;     // [2] scores of half h in TMEM
  uint64_t* p_full = bars + 3 + 2 * kRing;     // [2] half h's P / dS written back to TMEM (8 warps)
  uint64_t* acc_done = bars + 5 + 2 * kRing;
  uint64_t* drain = bars + 6 + 2 * kRing;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7 + 2 * kRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // KV kernel: per compute warp, its 32 columns' (-LSE log2 e, Delta) pairs.
  __shared__ __align__(16) float2 col_stats[kComputeWarps][32];

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
  // TMEM: accumulators at 0 (dV or dQ) and 128 (dK); half h's scores at
  // s_base + 128 h, its dP 64 columns further.
  constexpr uint32_t s_base = MODE == kModeKV ? 256u : 128u;

  if (threadIdx.x == 0) {
    mbar_init(res_full, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&ring_full[s], 1);
      mbar_init(&ring_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], kComputeWarps);
    }
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
      for (int u = 0; u < 2 * n_it; ++u) {
        const int st = u % kRing;
        const uint32_t ph = (uint32_t)(u / kRing) & 1u;
        if (!wait_bounded(&ring_empty[st], ph ^ 1u, wc, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        const int row0 = (it0 + (u >> 1)) * kB + (u & 1) * 64;
        uint8_t* dst = sRing + st * kHS;
        mbar_arrive_expect_tx(&ring_full[st], kHS);
        for (int h = 0; h < 2; ++h) {
          tma_load_4d(dst + h * 8192, s0, &ring_full[st], h * 64, row0, hi, bi);
          tma_load_4d(dst + 16384 + h * 8192, s1, &ring_full[st], h * 64, row0, hi, bi);
        }
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      drain_wait(res_full, 0, p.timeout_ns, p.err_word);
      if (!ok)
        for (int s = 0; s < kRing; ++s)
          if (armed & (1u << s)) drain_wait(&ring_full[s], (armed_par >> s) & 1u, p.timeout_ns, p.err_word);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc(1, 1, 1, 0, 0, 128, 64);   // scores of a half: N = 64
      constexpr uint32_t idesc_g = make_idesc(1, 1, 1, 0, 1, 128, 128);  // A from TMEM, B MN-major, N = 128
      const uint32_t res = smem_u32(sRes), ring = smem_u32(sRing);
      auto stage = [&](int u) { return ring + (uint32_t)((u % kRing) * kHS); };
      auto landed = [&](int u) {
        return wait_bounded(&ring_full[u % kRing], (uint32_t)(u / kRing) & 1u, wc, kErrTimeoutMma);
      };
      // Half h of streamed block t: scores (A resident, K-major; B the half's
      // 64 streamed rows, K-major) and dP likewise.
      auto scores = [&](int t, int h) {
        const uint32_t st = stage(2 * t + h);
        const uint32_t d_s = tmem + s_base + 128 * h;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) mma_ss<0>(d_s, kmajor(res, kk), kmajor_h(st, kk), idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ss<0>(d_s + 64, kmajor(res + kTile, kk), kmajor_h(st + 16384, kk), idesc_s, kk > 0 ? 1u : 0u);
        mma_commit(&s_full[h]);
      };
      bool ok = wait_bounded(res_full, 0, wc, kErrTimeoutMma) && landed(0);
      if (ok) {
        tc_fence_after();
        scores(0, 0);
        ok = landed(1);
        if (ok) {
          tc_fence_after();
          scores(0, 1);
        }
      }
      for (int t = 0; t < n_it && ok; ++t) {
        for (int h = 0; h < 2 && ok; ++h) {
          if (!wait_bounded(&p_full[h], t & 1, wc, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sh = tmem + s_base + 128 * h;
          const uint32_t st = stage(2 * t + h);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t acc = (t > 0 || h > 0 || kk > 0) ? 1u : 0u;
            if (MODE == kModeKV) {
              // dV += P^T dO_h, dK += dS^T Q_h (M = keys, K = this half's 64 queries)
              mma_ts_f16(tmem, sh + half_col(kk), mnmajor_h(st + 16384, kk), idesc_g, acc);
              mma_ts_f16(tmem + 128, sh + 64 + half_col(kk), mnmajor_h(st, kk), idesc_g, acc);
            } else {
              // dQ += dS_h K_h (M = queries, K = this half's 64 keys)
              mma_ts_f16(tmem, sh + half_col(kk), mnmajor_h(st, kk), idesc_g, acc);
            }
          }
          mma_commit(&ring_empty[(2 * t + h) % kRing]);
          if (t + 1 < n_it) {
            // In-order execution: the next scores land after the MMAs above
            // have read this half's columns.
            if (!landed(2 * (t + 1) + h)) {
              ok = false;
              break;
            }
            tc_fence_after();
            scores(t + 1, h);
          }
        }
      }
      mma_commit(acc_done);
      // Every MMA this thread issued must complete before TMEM is released.
      mma_commit(drain);
      drain_wait(drain, 0, p.timeout_ns, p.err_word);
    }
  } else {
    // ------------------------------------------------------------ P / dS and the epilogue
    const int q = warp & 3;
    const int sub = (warp - 2) >> 2;  // which 32 of a half's 64 columns
    const int row = q * 32 + lane;
    const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16);
    const long long stat_base = (long long)bh * p.seq_q;
    // Rows: KV keys of block `own`; Q queries of block `own`.
    const int rabs = own * kB + row;
    float row_lse = 0.f, row_dlt = 0.f;
    if (MODE == kModeQ && rabs < p.seq_q) {
      row_lse = p.lse[stat_base + rabs] * kLog2e;
      row_dlt = p.delta[stat_base + rabs];
    }
    bool ok = true;
    for (int t = 0; t < n_it && ok; ++t) {
      const int blk = it0 + t;  // streamed block (KV: query block, Q: key block)
      for (int h = 0; h < 2; ++h) {
        const int cbase = blk * kB + h * 64 + sub * 32;  // first column index (query or key)
        float col_lse = 0.f, col_dlt = 0.f;
        if (MODE == kModeKV && cbase + lane < p.seq_q) {
          col_lse = p.lse[stat_base + cbase + lane] * kLog2e;
          col_dlt = p.delta[stat_base + cbase + lane];
        }
        if (MODE == kModeKV) {
          __syncwarp();  // the previous half's reads of the slot are done
          col_stats[warp - 2][lane] = make_float2(-col_lse, col_dlt);
          __syncwarp();
        }
        if (!wait_bounded(&s_full[h], t & 1, wc, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t scol = s_base + 128 * h + 32 * sub;
        uint32_t rs[32], rd[32];
        tmem_ld_32x32b_x32(t_row + scol, rs);
        tmem_ld_32x32b_x32(t_row + scol + 64, rd);
        tmem_ld_wait();
        // The mask matters only on the causal diagonal and past the sequence
        // ends; every other (warp, half) block skips the per-element test.
        const int rlo = own * kB + q * 32, clo = cbase;  // this warp's first row / column
        bool all_valid;
        if (MODE == kModeKV)  // rows keys [rlo, rlo + 32), columns queries [clo, clo + 32)
          all_valid = rlo + 32 <= p.seq_k && clo + 32 <= p.seq_q && (!p.causal || rlo + 31 <= clo);
        else  // rows queries, columns keys
          all_valid = rlo + 32 <= p.seq_q && clo + 32 <= p.seq_k && (!p.causal || clo + 31 <= rlo);
        uint32_t pp[16], dd[16];
        if (all_valid) {
          // Packed pairs: x = S scale log2e - LSE log2e, P = 2^x, dS = P (dP - Delta).
          const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
          const uint64_t nl_row = f2_pack(-row_lse, -row_lse), nd_row = f2_pack(-row_dlt, -row_dlt);
          const float4* st4 = reinterpret_cast<const float4*>(col_stats[warp - 2]);
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2) {
            uint64_t nl2, nd2;
            if (MODE == kModeKV) {
              const float4 cs = st4[jj / 2];  // (-lse, dlt) of columns jj, jj + 1 (a broadcast load)
              nl2 = f2_pack(cs.x, cs.z);
              nd2 = f2_pack(-cs.y, -cs.w);
            } else {
              nl2 = nl_row;
              nd2 = nd_row;
            }
            const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(rs[jj]), __uint_as_float(rs[jj + 1])), sc2, nl2);
            float x0, x1;
            f2_unpack(x2, x0, x1);
            // Every kPolyEveryBwd-th pair on the FMA pipe, the rest on the SFU.
            const bool poly = kPolyEveryBwd > 0 && (jj / 2) % kPolyEveryBwd == kPolyEveryBwd - 1;
            const uint64_t p2 = poly ? f2_pack(exp2_poly(x0), exp2_poly(x1)) : f2_pack(ex2_approx(x0), ex2_approx(x1));
            const uint64_t d2 =
                f2_mul(p2, f2_add(f2_pack(__uint_as_float(rd[jj]), __uint_as_float(rd[jj + 1])), nd2));
            float p0, p1, d0, d1;
            f2_unpack(p2, p0, p1);
            f2_unpack(d2, d0, d1);
            pp[jj / 2] = pack_bf16(p0, p1);
            dd[jj / 2] = pack_bf16(d0, d1);
          }
        } else
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          float pv[2], dv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = cbase + jj + e;
            float lse_l2, dlt;
            bool valid = true;
            if (MODE == kModeKV) {  // row = key rabs, column = query c
              lse_l2 = __shfl_sync(0xffffffffu, col_lse, jj + e);
              dlt = __shfl_sync(0xffffffffu, col_dlt, jj + e);
              if (!all_valid) valid = c < p.seq_q && rabs < p.seq_k && (!p.causal || rabs <= c);
            } else {  // row = query rabs, column = key c
              lse_l2 = row_lse;
              dlt = row_dlt;
              if (!all_valid) valid = rabs < p.seq_q && c < p.seq_k && (!p.causal || c <= rabs);
            }
            pv[e] = valid ? ex2_approx(fmaf(__uint_as_float(rs[jj + e]), p.scale_log2, -lse_l2)) : 0.f;
            dv[e] = pv[e] * (__uint_as_float(rd[jj + e]) - dlt);
          }
          pp[jj / 2] = pack_bf16(pv[0], pv[1]);
          dd[jj / 2] = pack_bf16(dv[0], dv[1]);
        }
        // This warp's 32 columns, packed, over its own scores (P) and dP (dS).
        if (MODE == kModeKV) {
          tmem_st_32x32b_x16(t_row + scol, pp);
          tmem_st_32x32b_x16(t_row + scol + 64, dd);
        } else {
          tmem_st_32x32b_x16(t_row + scol, dd);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[h]);
      }
    }
    if (ok && wait_bounded(acc_done, 0, wc, kErrTimeoutEpilogue) && !*abort_flag) {
      tc_fence_after();
      // KV: dK (scaled) from [128, 256) to out0, dV from [0, 128) to out1.
      // Q: dQ (scaled) from [0, 128) to out0. Warp sub writes columns [64 sub, +64).
      const bool rvalid = rabs < (MODE == kModeKV ? p.seq_k : p.seq_q);
      for (int which = 0; which < (MODE == kModeKV ? 2 : 1); ++which) {
        const uint32_t col = MODE == kModeKV ? (which == 0 ? 128u : 0u) : 0u;
        const float mul = which == 0 ? p.scale : 1.f;
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(which == 0 ? p.out0 : p.out1) +
                             (which == 0 ? (long long)bi * p.o0_sb + (long long)hi * p.o0_sh + (long long)rabs * p.o0_ss
                                         : (long long)bi * p.o1_sb + (long long)hi * p.o1_sh + (long long)rabs * p.o1_ss);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int c0 = sub * 64 + c * 32;
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + col + c0, v);
          tmem_ld_wait();
          if (rvalid) {
            uint4* dst = reinterpret_cast<uint4*>(out + c0);
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

// [batch, heads, seq, 128] bf16 -> 4-D map {128, seq, heads, batch}, box {64, box_rows, 1, 1}
// (128 rows for a resident tile, 64 for a streamed half-block).
// A batch or head stride of 0 (broadcast) is replaced by the dense stride the
// map needs for a dimension of extent 1.
bool make_map(CUtensorMap* m, const void* base, int batch, int heads, int seq, long long sb, long long sh,
              long long ss, int box_rows) {
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
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
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
  // Resident tiles (KV kernel: K, V; Q kernel: Q, dO) are loaded as 128-row
  // boxes, streamed half-blocks as 64-row boxes.
  CUtensorMap mq[2], mk[2], mv[2], md[2];  // [0]: 128-row boxes, [1]: 64-row boxes
  for (int i = 0; i < 2; ++i) {
    const int rows = i == 0 ? 128 : 64;
    if (!make_map(&mq[i], a.q, a.batch, a.heads, a.seq_q, a.q_sb, a.q_sh, a.q_ss, rows) ||
        !make_map(&mk[i], a.k, a.batch, a.heads, a.seq_k, a.k_sb, a.k_sh, a.k_ss, rows) ||
        !make_map(&mv[i], a.v, a.batch, a.heads, a.seq_k, a.v_sb, a.v_sh, a.v_ss, rows) ||
        !make_map(&md[i], a.dout, a.batch, a.heads, a.seq_q, a.do_sb, a.do_sh, a.do_ss, rows))
      return cudaErrorNotSupported;
  }
  const void* outs[3] = {a.dq, a.dk, a.dv};
  const long long oss[3] = {a.dq_ss, a.dk_ss, a.dv_ss};
  for (int i = 0; i < 3; ++i)
    if ((reinterpret_cast<uintptr_t>(outs[i]) & 15u) || (oss[i] * 2) % 16) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(a.o) & 15u) || (reinterpret_cast<uintptr_t>(a.dout) & 15u) || (a.o_ss * 2) % 16 ||
      (a.do_ss * 2) % 16 || (a.o_sh * 2) % 16 || (a.o_sb * 2) % 16 || (a.do_sh * 2) % 16 || (a.do_sb * 2) % 16)
    return cudaErrorNotSupported;
  float* delta = static_cast<float*>(ws);
  {
    const long long rows = (long long)a.batch * a.heads * a.seq_q;
    const long long blocks = (rows + 15) / 16;  // 256 threads = 16 rows
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
  cudaError_t e = launch_mode<kModeKV>(mq[1], mk[0], mv[0], md[1], p, s);
  if (e != cudaSuccess) return e;
  p.out0 = a.dq;
  p.o0_sb = a.dq_sb; p.o0_sh = a.dq_sh; p.o0_ss = a.dq_ss;
  p.out1 = nullptr;
  return launch_mode<kModeQ>(mq[0], mk[1], mv[1], md[0], p, s);
}

}  // namespace grx
