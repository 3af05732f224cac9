/*
 * ref_binlayer_harness.c -- thin C shim over the REFERENCE's own BinLayer code.
 *
 * TEST INFRASTRUCTURE ONLY.  Linked (by oracle/Makefile, target `ref`) against
 * the reference's runtime/lal_runtime.c compiled from its source tree; the
 * result lands in oracle/_ref/liblal_ref.so and is used to produce the golden
 * fixtures for the seed STE model's logic-masked forward.
 *
 * It builds a BinLayer exactly as the reference's model_load does for a
 * logic-masked layer (bin_layer_init_logic, runtime/lal_runtime.c:1567-1676),
 * optionally re-derives alpha with bin_layer_repack (:1703-1766), and runs
 *   bin_forward            (:1852-1956, mode 0)  or
 *   bin_forward_pure_float (:543-582,   mode 1)
 * once per input row.  Globals the forward reads are set explicitly:
 * g_binary_scale (:663), g_use_ternary, g_use_cuda.
 */
#include "lal_runtime.h"

#include <string.h>

int lalref_binlayer_forward(const float *W, const float *bias,
                            const uint8_t *mask, int in_dim, int out_dim,
                            const float *X, int M, float *Y, int mode,
                            int repack, float binary_scale, float *alpha_out) {
    BinLayer bl;
    memset(&bl, 0, sizeof(bl));
    g_use_ternary = 0;
    g_use_cuda = 0;
    g_binary_scale = binary_scale;
    bin_layer_init_logic(&bl, W, bias, in_dim, out_dim, mask);
    if (repack) bin_layer_repack(&bl);
    if (alpha_out) memcpy(alpha_out, bl.alpha, sizeof(float) * out_dim);
    for (int m = 0; m < M; m++) {
        const float *x = X + (size_t)m * in_dim;
        float *y = Y + (size_t)m * out_dim;
        if (mode == 0)
            bin_forward(y, x, &bl);
        else
            bin_forward_pure_float(y, x, &bl);
    }
    bin_layer_free(&bl);
    return 0;
}
