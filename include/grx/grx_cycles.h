/* grxcp-b200 -- per-CTA timing probe ABI.
 *
 * Same record as the reference's cycle probe (include/grx/grx_cycles.h:39-44):
 * the kernel writes one slot per unit of work. On B200 a slot is one CTA of the
 * sgemm kernel; `start`/`end` are the SM's clock64() counter, `core` is the SM
 * id (%smid) and `warp` the CTA's linear index.
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

#ifdef __cplusplus
}
#endif

#endif /* GRX_CYCLES_H */
