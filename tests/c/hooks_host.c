/*
 * A C host that puts the B200 linear leaf under the reference's own engine
 * (test build; linked against the reference engine compiled from its
 * sources and against libapus_gcuda.so).
 *
 * The reference dispatches every BF16 GEMM/GEMV (c/bf16.h:717-744) and every
 * fused FP8-block linear (c/gdsa.h:529-530) through its global hook table
 * apus_gmetal_hooks (c/backend_gmetal.h:120-128); the Metal backend fills it
 * on macOS.  apus_gcuda_fill_hooks fills the same layout.  This is the whole
 * integration: the engine itself is not edited.
 */
#include <stdint.h>
#include <string.h>

#include "apus_gcuda.h"

/* the reference's table (ApusGmetalHooks: the same two function pointers) */
extern ApusGcudaHooks apus_gmetal_hooks;

int host_attach(char *err, size_t errcap) {
    if (apus_gcuda_enable(err, errcap)) return -1;
    ApusGcudaHooks h;
    apus_gcuda_fill_hooks(&h);
    memcpy(&apus_gmetal_hooks, &h, sizeof h);
    return 0;
}

void host_detach(void) { memset(&apus_gmetal_hooks, 0, sizeof apus_gmetal_hooks); }

int host_attached(void) { return apus_gmetal_hooks.bf16_gemm != NULL && apus_gmetal_hooks.fp8blk_linear != NULL; }
