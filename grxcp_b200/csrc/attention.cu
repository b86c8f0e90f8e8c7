// Fused scaled-dot-product attention forward for sm_100a (grxDNN; the
// reference plans "fused attention" at docs/designs/grxcp_roadmap.md:864-865
// and implements none).
//
// One CTA per (batch, head, pair of 128-query tiles); causal grids launch the
// longest pairs first. 320 threads:
//   warp 0      TMA producer: both Q tiles once, then K_0, V_0, K_1, V_1, ...
//               (128 keys x 128 dims bf16, 128-byte swizzle) through a 4-slot
//               ring of 32 KiB.
//   warp 1      MMA issuer (one thread). Per key block j, per query tile i:
//               S_i = Q_i K_j^T into TMEM (SS MMA), then O_i += P_i V_j with P_i
//               read straight from TMEM (TS MMA). The issue order
//               PV_0(j), QK_0(j+1), PV_1(j), QK_1(j+1) lets the tensor core
//               work on one tile while the other tile's softmax runs.
//   warps 2..5  softmax of tile 0, warps 6..9 softmax of tile 1 (thread =
//               query row): read S from TMEM, mask (diagonal and ragged blocks
//               only), online max/sum in the exp2 domain with the softmax scale
//               folded into one FFMA, ex2 on the SFU, write P as packed bf16
//               pairs back over S's TMEM columns; rescale O in TMEM only when
//               the running max grows by more than 2^8; finally normalise O,
//               store bf16 O and the fp32 natural-log LSE.
// TMEM: S0 [0,128), S1 [128,256), O0 [256,384), O1 [384,512). P_i occupies
// the first 64 columns of S_i; QK_i(j+1) overwrites them only after PV_i(j),
// and tcgen05.mma ops from one thread execute in issue order.
// All waits are bounded (ptx.cuh).
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "attention.cuh"
#include "exp2_poly.cuh"
#include "ptx.cuh"
#include "profile.h"

namespace grx {

namespace {

constexpr int kD = 128;                   // head dim
constexpr int kBQ = 128;                  // queries per tile (two tiles per CTA)
constexpr int kBK = 128;                  // keys per block
constexpr int kTileBytes = 128 * kD * 2;  // one 128 x 128 bf16 tile = 32 KiB (two 16 KiB swizzle halves)
constexpr int kHalf = 16384;
constexpr int kSlots = 4;                 // K/V ring slots
constexpr int kThreads = 320;
constexpr int kSmem = 2 * kTileBytes /*Q0,Q1*/ + kSlots * kTileBytes + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kPolyEvery = 8;              // every 8th pair of exponentials on the FMA pipe (measured best of 2/4/8/none)
constexpr int kHeadGroup = 16;             // (batch, head) pairs scheduled together (K/V stay in L2)

struct AttnParams {
  int batch, heads, seq_q, seq_k, n_qp, n_kb, causal;
  float scale_log2;
  void* o;
  long long o_sb, o_sh, o_ss;
  float* lse;
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

// K-major operand descriptor for a 128-row x 128-element (bf16) tile stored as
// two 64-element swizzle halves; kk selects the 16-element k slice.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return sw128_desc(base + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}

// Packed fp32 pairs (sm_100 executes f32x2 FMA/ADD as one instruction).
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&s)[128]) {
  uint32_t u[4][32];
  tmem_ld_32x32b_x32(taddr + 0, u[0]);
  tmem_ld_32x32b_x32(taddr + 32, u[1]);
  tmem_ld_32x32b_x32(taddr + 64, u[2]);
  tmem_ld_32x32b_x32(taddr + 96, u[3]);
  tmem_ld_wait();
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(u[c][e]);
}

// 10 warps: three of them share an SM sub-partition's 16K-register file, which
// caps the kernel at 168 registers per thread.
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;                     // Q0 at 0, Q1 at kTileBytes
  uint8_t* sKV = sQ + 2 * kTileBytes;     // slot s at s * kTileBytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kSlots * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* slot_full = bars + 1;
  uint64_t* slot_empty = slot_full + kSlots;
  uint64_t* s_full = slot_empty + kSlots;  // [2]
  uint64_t* p_full = s_full + 2;           // [2]
  uint64_t* o_done = p_full + 2;           // [2]
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA order: groups of kHeadGroup (batch, head) pairs, and within a group
  // every query-tile pair of those heads, longest causal pairs first -- so the
  // K/V of a group (2 MiB per head at S = 4096) stay in L2 while all of its
  // query tiles pass over them.
  const int bh_count = p.batch * p.heads;
  const int full_groups = bh_count / kHeadGroup;
  const int idx = blockIdx.x;
  int g, w, gsz;
  if (idx < full_groups * kHeadGroup * p.n_qp) {
    g = idx / (kHeadGroup * p.n_qp);
    w = idx - g * kHeadGroup * p.n_qp;
    gsz = kHeadGroup;
  } else {
    g = full_groups;
    w = idx - full_groups * kHeadGroup * p.n_qp;
    gsz = bh_count - full_groups * kHeadGroup;
  }
  const int qrank = w / gsz;
  const int bh = g * kHeadGroup + (w - qrank * gsz);
  const int qp = p.causal ? (p.n_qp - 1 - qrank) : qrank;
  const int bi = bh / p.heads, hi = bh % p.heads;
  // key blocks each query tile needs
  int nblk[2];
  nblk[0] = p.causal ? min(2 * qp + 1, p.n_kb) : p.n_kb;
  nblk[1] = p.causal ? min(2 * qp + 2, p.n_kb) : p.n_kb;
  const int nall = max(nblk[0], nblk[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&slot_full[s], 1);
      mbar_init(&slot_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);
      mbar_init(&o_done[b], 1);
    }
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
  const uint32_t tmem = *tmem_slot;
  WaitCtx wc{p.err_word, abort_flag, p.timeout_ns};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      for (int t = 0; t < 2; ++t) {
        tma_load_4d(sQ + t * kTileBytes, &tmQ, q_full, 0, (2 * qp + t) * kBQ, hi, bi);
        tma_load_4d(sQ + t * kTileBytes + kHalf, &tmQ, q_full, 64, (2 * qp + t) * kBQ, hi, bi);
      }
      for (int L = 0; L < 2 * nall && ok; ++L) {
        const int slot = L % kSlots;
        const uint32_t ph = (L / kSlots) & 1;
        if (!wait_bounded(&slot_empty[slot], ph ^ 1u, wc, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        const CUtensorMap* m = (L & 1) ? &tmV : &tmK;
        uint8_t* dst = sKV + slot * kTileBytes;
        mbar_arrive_expect_tx(&slot_full[slot], kTileBytes);
        tma_load_4d(dst, m, &slot_full[slot], 0, (L >> 1) * kBK, hi, bi);
        tma_load_4d(dst + kHalf, m, &slot_full[slot], 64, (L >> 1) * kBK, hi, bi);
        armed |= 1u << slot;
        armed_par = (armed_par & ~(1u << slot)) | (ph << slot);
      }
      drain_wait(q_full, 0, p.timeout_ns, p.err_word);
      if (!ok)
        for (int s = 0; s < kSlots; ++s)
          if (armed & (1u << s)) drain_wait(&slot_full[s], (armed_par >> s) & 1u, p.timeout_ns, p.err_word);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc(1, 1, 1, 0, 0, 128, 128);  // bf16, both K-major
      constexpr uint32_t idesc_o = make_idesc(1, 1, 1, 0, 1, 128, 128);  // A (P, TMEM) K-major, V MN-major
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = wait_bounded(q_full, 0, wc, kErrTimeoutMma);
      tc_fence_after();
      auto slot_of = [](int L) { return L % kSlots; };
      auto par_of = [](int L) { return (uint32_t)((L / kSlots) & 1); };
      auto qk = [&](int t, int j) {
        const uint32_t k_addr = smem_u32(sKV + slot_of(2 * j) * kTileBytes);
        const uint32_t qa = q_addr + t * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ss<0>(tmem + t * 128, kmajor_desc(qa, kk), kmajor_desc(k_addr, kk), idesc_s, kk > 0 ? 1u : 0u);
        mma_commit(&s_full[t]);
      };
      auto pv = [&](int t, int j) {
        const uint32_t v_addr = smem_u32(sKV + slot_of(2 * j + 1) * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts_f16(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, sw128_desc(v_addr + kk * 2048, kHalf, 1024),
                     idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&o_done[t]);
      };
      // block 0 scores for both tiles
      if (ok && wait_bounded(&slot_full[slot_of(0)], par_of(0), wc, kErrTimeoutMma)) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (nblk[t] > 0) qk(t, 0);
        mma_commit(&slot_empty[slot_of(0)]);
      } else {
        ok = false;
      }
      for (int j = 0; j < nall && ok; ++j) {
        if (!wait_bounded(&slot_full[slot_of(2 * j + 1)], par_of(2 * j + 1), wc, kErrTimeoutMma)) break;
        const bool next = j + 1 < nall;
        bool k_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j < nblk[t]) {
            if (!wait_bounded(&p_full[t], j & 1, wc, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            pv(t, j);
          }
          if (next && j + 1 < nblk[t]) {
            if (!k_ready) {
              if (!wait_bounded(&slot_full[slot_of(2 * j + 2)], par_of(2 * j + 2), wc, kErrTimeoutMma)) {
                ok = false;
                break;
              }
              tc_fence_after();
              k_ready = true;
            }
            qk(t, j + 1);
          }
        }
        if (!ok) break;
        mma_commit(&slot_empty[slot_of(2 * j + 1)]);      // V_j done
        if (next) mma_commit(&slot_empty[slot_of(2 * j + 2)]);  // K_{j+1} done (or unused)
      }
      mma_commit(drain);
      drain_wait(drain, 0, p.timeout_ns, p.err_word);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = (warp - 2) >> 2;         // query tile 0 (warps 2-5) or 1 (warps 6-9)
    const int qd = warp & 3;               // TMEM lane quadrant this warp may access
    const int r = qd * 32 + lane;
    const int q0 = (2 * qp + t) * kBQ;     // first query of this tile
    const int qi = q0 + r;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + t * 128;
    const uint32_t o_addr = tmem + lane_base + 256 + t * 128;
    const int nb = nblk[t];
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      if (!wait_bounded(&s_full[t], j & 1, wc, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
      tmem_ld4(s_addr, s);

      const int key0 = j * kBK;
      const bool need_mask = (key0 + kBK > p.seq_k) || (p.causal && key0 + kBK - 1 > q0);
      if (need_mask) {
        const int lim = p.causal ? min(qi + 1, p.seq_k) : p.seq_k;  // keys < lim are visible
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (key0 + c >= lim) s[c] = -INFINITY;
      }
      // Row max: eight independent 3-input max chains (0.5 instructions per score).
      float mx[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx[u] = fmaxf(s[2 * u], s[2 * u + 1]);
#pragma unroll
      for (int c = 16; c < 128; c += 16)
#pragma unroll
        for (int u = 0; u < 8; ++u) mx[u] = max3(mx[u], s[c + 2 * u], s[c + 2 * u + 1]);
      const float mb = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
      const float m_blk = mb * p.scale_log2;  // scale > 0: max commutes with scaling
      const float m_new = fmaxf(m_run, m_blk);
      const bool rescale = (j == 0) || (m_new > m_run + kRescaleThreshold);
      float m_use = rescale ? m_new : m_run;
      if (m_use == -INFINITY) m_use = 0.f;
      const float alpha = (rescale && j > 0) ? ex2_approx(m_run - m_use) : 1.f;
      // x = s * scale*log2(e) - m as packed pairs, 2^x, packed running sums.
      const uint64_t sc2 = pack2(p.scale_log2, p.scale_log2);
      const uint64_t nm2 = pack2(-m_use, -m_use);
      uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        float x0, x1;
        unpack2(ffma2(pack2(s[c], s[c + 1]), sc2, nm2), x0, x1);
        // One pair in kPolyEvery goes to the FMA pipe, the rest to the SFU.
        const bool poly = ((c >> 1) % kPolyEvery) == kPolyEvery - 1;
        const float p0 = poly ? exp2_poly(x0) : ex2_approx(x0);
        const float p1 = poly ? exp2_poly(x1) : ex2_approx(x1);
        acc[(c >> 1) & 3] = fadd2(acc[(c >> 1) & 3], pack2(p0, p1));
        __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
        pk[c >> 1] = *reinterpret_cast<uint32_t*>(&h);
      }
      float a0, a1, a2, a3, a4, a5, a6, a7;
      unpack2(acc[0], a0, a1);
      unpack2(acc[1], a2, a3);
      unpack2(acc[2], a4, a5);
      unpack2(acc[3], a6, a7);
      const float rs = ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7));
      l_run = l_run * alpha + rs;
      m_run = m_use;

      if (j > 0) {
        // PV of the previous block must be done: it reads P (over S) and writes O.
        if (!wait_bounded(&o_done[t], (j - 1) & 1, wc, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t u[32];
            tmem_ld_32x32b_x32(o_addr + c * 32, u);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
            tmem_st_32x32b_x32(o_addr + c * 32, u);
          }
        }
      }
      uint32_t (&pk0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[0]);
      uint32_t (&pk1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[32]);
      tmem_st_32x32b_x32(s_addr, pk0);
      tmem_st_32x32b_x32(s_addr + 32, pk1);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok && nb > 0 && wait_bounded(&o_done[t], (nb - 1) & 1, wc, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.o) + (long long)bi * p.o_sb + (long long)hi * p.o_sh +
                            (long long)qi * p.o_ss;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(o_addr + c * 32, u);
        tmem_ld_wait();
        if (qi < p.seq_q) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(u[e + 2 * q]) * inv_l,
                                                       __uint_as_float(u[e + 2 * q + 1]) * inv_l);
              wp[q] = *reinterpret_cast<uint32_t*>(&h);
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
  p.n_qp = (a.seq_q + 2 * kBQ - 1) / (2 * kBQ);
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
  const long long grid = (long long)p.n_qp * a.batch * a.heads;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  });
  if (attr != cudaSuccess) return attr;
  ProfLaunch prof("attn_fwd_kernel", dim3((unsigned)grid), dim3(kThreads), kSmem, s);
  attn_fwd_kernel<<<(unsigned)grid, kThreads, kSmem, s>>>(mq, mk, mv, p);
  return cudaGetLastError();
}

}  // namespace grx
