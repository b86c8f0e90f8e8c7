/* grxcp-b200 -- per-CTA timing probe ABI.
 *
 * Same record as the reference's cycle probe (include/grx/grx_cycles.h:39-54):
 * the kernel writes one slot per unit of work. On B200 a slot is one CTA of the
 * sgemm kernel or of the tensor-core GEMM; `start`/`end` are the SM's clock64()
 * counter, `core` is the SM id (%smid) and `warp` the CTA's linear index.
 *
 * clock64() counts cycles of one SM and the SMs' counters are not aligned with
 * one another, so a span (first start to last end) is only meaningful when every
 * written slot came from one SM. grxCycleSummarize then reports it; otherwise it
 * says the span is invalid instead of returning a number (reference
 * grx_cycles.h:20-27).
 */
#ifndef GRX_CYCLES_H
#define GRX_CYCLES_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  uint64_t start;
  uint64_t end;
  uint32_t core;
  uint32_t warp;
} grxCycleSlot;

/* reference grx_cycles.h:46-54 */
typedef struct {
  int      warps;        /* slots that were written (start or end non-zero) */
  int      cores;        /* 1 when they all came from one SM, else 2 */
  int      spanIsValid;  /* 1 only when cores == 1 */
  uint64_t span;         /* latest end - earliest start, 0 when invalid */
  uint64_t busyMin;      /* per-slot end - start: minimum, median, maximum */
  uint64_t busyMedian;
  uint64_t busyMax;
} grxCycleSummary;

#ifdef __cplusplus
}
#endif

#if defined(__cplusplus) && !defined(__CUDA_ARCH__)
#include <algorithm>
#include <vector>

/* Host-only summary of a probe array (behaviour of reference grx_cycles.h:67-99):
 * slots left all-zero were never reached by a CTA and are skipped; the median is
 * the element at index count/2 of the sorted busy times. */
inline void grxCycleSummarize(const grxCycleSlot* slots, int n, grxCycleSummary* out) {
  if (out == nullptr) return;
  grxCycleSummary s = {};
  std::vector<uint64_t> busy;
  uint64_t lo = 0, hi = 0;
  uint32_t first_core = 0;
  bool single_sm = true;
  for (int i = 0; slots != nullptr && i < n; ++i) {
    const grxCycleSlot& r = slots[i];
    if (r.start == 0 && r.end == 0) continue;
    if (busy.empty()) {
      lo = r.start;
      hi = r.end;
      first_core = r.core;
    } else {
      single_sm = single_sm && r.core == first_core;
      lo = r.start < lo ? r.start : lo;
      hi = r.end > hi ? r.end : hi;
    }
    busy.push_back(r.end - r.start);
  }
  if (!busy.empty()) {
    const size_t mid = busy.size() / 2;
    std::nth_element(busy.begin(), busy.begin() + mid, busy.end());
    s.busyMedian = busy[mid];
    s.busyMin = *std::min_element(busy.begin(), busy.end());
    s.busyMax = *std::max_element(busy.begin(), busy.end());
    s.warps = (int)busy.size();
    s.cores = single_sm ? 1 : 2;
    s.spanIsValid = single_sm ? 1 : 0;
    s.span = single_sm ? hi - lo : 0;
  }
  *out = s;
}
#endif

#endif /* GRX_CYCLES_H */
