/* grxcp-b200 -- tensor-map declarations of the GRXCP runtime.
 *
 * Names, fields and enum values are the reference's (include/grx/grx_tensormap.h
 * :37-120 in kubeworkz/grxcp), because the reference grxblas.h includes this
 * header and callers may name its types.
 *
 * On B200 a TMA descriptor (CUtensorMap) is a 128-byte value built per launch
 * and passed in the kernel's parameter block; the device has no descriptor
 * slots to program. This library's kernels build their own descriptors, so:
 *   grxTensorMapGetSlotCount   reports 0 slots (success)
 *   grxTensorMapProgram(Async) returns grxErrorNotSupported (nothing to program)
 *   grxMallocPhysical          is grxMalloc: TMA goes through the same address
 *                              translation as every other access on this GPU.
 */
#ifndef GRX_TENSORMAP_H
#define GRX_TENSORMAP_H

#include "grx_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* reference grx_tensormap.h:43-52 */
typedef enum {
  grxTensorMapLayoutRowMajor = 0,
  grxTensorMapLayoutKMajor   = 1
} grxTensorMapLayout_t;

/* reference grx_tensormap.h:61-74: sizes and tiles in elements, strides in bytes. */
typedef struct {
  int      slot;
  void*    base;
  unsigned rank;
  unsigned size[5];
  unsigned strideBytes[4];
  unsigned tile[5];
  unsigned elementBytes;
  grxTensorMapLayout_t layout;
  unsigned smemStrideBytes;
} grxTensorMapDesc_t;

/* reference grx_tensormap.h:78 */
grxError_t grxTensorMapGetSlotCount(int* count, int device);
/* reference grx_tensormap.h:96 */
grxError_t grxMallocPhysical(void** ptr, size_t size);
/* reference grx_tensormap.h:106-108 */
grxError_t grxTensorMapProgramAsync(const grxTensorMapDesc_t* desc, grxStream_t stream);
grxError_t grxTensorMapProgram(const grxTensorMapDesc_t* desc);

#ifdef __cplusplus
}
#endif

#endif /* GRX_TENSORMAP_H */
