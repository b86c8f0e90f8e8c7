/* grxcp-b200 -- umbrella header for host code.
 *
 * Same umbrella as the reference's include/grx/grx.h:5-7 (types, the runtime
 * subset, tensor-map declarations), so a reference caller that starts with
 * `#include <grx/grx.h>` compiles against this tree unchanged.
 */
#ifndef GRX_H
#define GRX_H

#include "grx_types.h"
#include "grx_runtime.h"
#include "grx_tensormap.h"

#endif /* GRX_H */
