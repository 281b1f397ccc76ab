/*
 * apus_gmoe_gcuda.h — the GLM-5.3-Flash MoE sublayer (c/gmoe.h) on the B200.
 *
 * The reference passes per-call host views of dequantized BF16 experts
 * (ApusGmoeW, c/gmoe.h:129-139).  The B200 layer instead keeps every expert
 * resident in HBM as FP8-E4M3 with its F32 128x128 block scales (the
 * north-star "full HBM residency" that replaces the NVMe expert cache), so
 * the weights are loaded once into an opaque object and each call only moves
 * activations.  Numerics follow c/gmoe.h:191-336: fp32 router, numpy-stable
 * sigmoid, selection-only bias, stable top-k with lower-index ties, weights
 * normalised with the numpy pairwise sum and scaled, SwiGLU with the limit
 * clamps, ascending-expert BF16 accumulation, shared expert last.  The
 * expert GEMVs keep the reference's BF16-rounded dequantized weights; only
 * fp32 summation orders differ (tolerance parity).  Selections are exact
 * whenever the router logits agree (they are fp32 dot products).
 */
#ifndef APUS_GMOE_GCUDA_H
#define APUS_GMOE_GCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ApusGcudaMoe ApusGcudaMoe;

/* A resident MoE sublayer: E routed experts of intermediate `inter` plus one
 * shared expert of the same width, top-k routing, hidden `dim`; max_rows
 * (<= 8) activation rows per call.  NULL on error (apus_gcuda_last_error). */
ApusGcudaMoe *apus_gcuda_moe_new(int E, int topk, size_t dim, size_t inter, float route_scale,
                                 float swiglu_limit, int max_rows);
void apus_gcuda_moe_free(ApusGcudaMoe *m);

/* Load one tensor by its checkpoint name (the names c/gmodel.h resolves):
 * "mlp.gate.weight" BF16 [E,dim], "mlp.gate.e_score_correction_bias" F32 [E],
 * "mlp.experts.<e>.{gate,up,down}_proj.weight" E4M3 and ".weight_scale_inv"
 * F32, "mlp.shared_experts.{gate,up,down}_proj.*".  A "layers.<l>." prefix is
 * accepted and ignored.  Host pointer, synchronous.  0 ok, -1 unknown name or
 * size mismatch. */
int apus_gcuda_moe_set(ApusGcudaMoe *m, const char *name, const void *host, size_t bytes);

/* Read one resident tensor back (same names and sizes as _set). */
int apus_gcuda_moe_get(ApusGcudaMoe *m, const char *name, void *host, size_t bytes);

/* Seeded synthetic weights with the BASELINE config-1 distributions: router
 * BF16 N(0, 0.02), bias 0, expert codes RNE-E4M3(N(0,1)*64), block scales
 * log-uniform in [1e-4, 1e-2].  Generated on the device. */
int apus_gcuda_moe_init_random(ApusGcudaMoe *m, uint64_t seed);

/* Device-pointer forward: x [s, dim] BF16 -> out [s, dim] BF16 on `stream`.
 * forced_idx: optional DEVICE [s, topk] selections (teacher forcing,
 * c/gmoe.h:145-152).  s <= max_rows. */
int apus_gcuda_moe_forward_dev(ApusGcudaMoe *m, const uint16_t *x, size_t s, uint16_t *out,
                               const int32_t *forced_idx, void *stream);

/* c/gmoe.h:153-155 apus_gmoe_forward2 with host buffers (interm/scratch
 * belong to the CPU engine and are ignored; forced_idx is a HOST array or
 * NULL).  Returns 0 ok, -1 error. */
int apus_gcuda_moe_forward2(ApusGcudaMoe *m, const uint16_t *x, size_t s, uint16_t *out,
                            const int32_t *forced_idx);

/* Routing of the last call (c/gmoe.h:112-117 router_idx / router_w): idx
 * [s, topk] in top-k order and w [s, topk] matching weights, host arrays. */
int apus_gcuda_moe_last_routing(ApusGcudaMoe *m, size_t s, int32_t *idx, float *w);

/* Weight bytes one call reads for the experts it selected (the algorithmic
 * bytes of the grouped GEMVs), from the last call's routing. */
uint64_t apus_gcuda_moe_last_bytes(ApusGcudaMoe *m);

#ifdef __cplusplus
}
#endif
#endif
