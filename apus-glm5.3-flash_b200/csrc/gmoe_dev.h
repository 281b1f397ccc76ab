// gmoe_dev.h — device-side MoE sublayer descriptor (internal).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define MOE_MAX_R 8
#define MOE_MAX_E 512
#define MOE_MAX_TOPK 16

#define EP_MAX_RANKS 8

// Expert-parallel exchange context (one process per GPU).  Every rank owns one
// exchange region, mapped into every peer through CUDA IPC:
//   contrib [2][MOE_MAX_R][MOE_MAX_TOPK][dim] BF16  weighted expert outputs
//   keys    [2][MOE_MAX_R] u64                      lm_head argmax keys
//   flags   [EP_MAX_RANKS] int                      barrier epochs, written by peers
// The [2] halves alternate with the barrier epoch's parity, so a rank never
// overwrites a half a peer may still be reading.  world == 1: no exchange.
struct EpCtx {
    int rank, world;
    uint8_t *peer[EP_MAX_RANKS];  // every rank's region (peer[rank] is this rank's)
    int *epoch;                   // this rank's exchange counter (device); epoch[1]: CTA arrivals
    long off_keys, off_flags;     // byte offsets inside a region
    // the prompt pass's weighted expert outputs [2][wide_rows][wide_k][dim]
    // BF16 (halves by epoch parity, as contrib), at off_wide
    long off_wide;
    int wide_rows, wide_k;
    // lm_head logits rows [MOE_MAX_R][V] BF16 at off_logits: each rank writes
    // its vocabulary slice's columns there, the others gather them
    long off_logits;
    int vocab;
};

// All pointers are device memory.  Weights: see gmoe.cu for the packed layout.
struct MoeDev {
    int E, topk, dim, inter, max_r, pdl;
    int e0, eloc;                 // this rank's routed experts [e0, e0+eloc); local slot eloc = shared
    EpCtx ep;
    float route_scale, limit;
    const uint16_t *gate_w;      // [E][dim] BF16 router
    const float *gate_bias;      // [E] f32 (selection-only bias)
    const uint8_t *gu_codes;     // [E+1][2*inter][dim] E4M3 (expert E = shared)
    const float *gu_scales;      // [E+1][2*inter/128][ceil(dim/128)]
    const uint8_t *d_codes;      // [E+1][dim][inter]
    const float *d_scales;       // [E+1][ceil(dim/128)][ceil(inter/128)]
    // per-call scratch
    float *logits;               // [max_r][E]
    int32_t *row_expert;         // [max_r][topk] selected experts, ascending
    float *row_weight;           // [max_r][topk] weights in that order
    int32_t *row_sel;            // [max_r][topk] selection in top-k order
    int32_t *row_prob;           // [max_r][topk] problem slot of each selection
    int32_t *row_prob_shared;    // [max_r] problem slot of the shared expert
    int32_t *prob_slot;          // [max_r*topk+1][8] selection slot j of (problem, row), -1: none
                                 // (expert parallelism only)
    int32_t *prob_expert;        // [max_r*topk+1] expert of each problem slot
    int32_t *prob_count;         // [1]
    unsigned long long *stat_problems;   // optional: += expert problems (incl. shared) per call
    float *part;                 // split-K scratch of the router GEMV (gemv_scratch_need(E, dim))
    int *tick;
    uint16_t *gu;                // [max_r*topk+1][max_r][2*inter]
    uint16_t *yd;                // [max_r*topk+1][max_r][dim]
};

// Buffers of the prompt pass's MoE over up to W rows: every row routed at
// once, then each active (local) expert's rows gathered into problems of 8
// rows, so an expert's weights stream once per 8 of its rows instead of once
// per 8 prompt rows.  pmax = W*topk/8 + E + W/8 + 1 problems.  With expert
// parallelism each rank runs its own experts' problems (pair_slot -1 for
// another rank's), writes the weighted outputs into its exchange region, and
// the combine reads them from their owners after one barrier.
struct MoeRows {
    int W, pmax;
    float *logits;          // [W][E] router logits (fp32)
    int32_t *row_expert;    // [W][topk] selections, ascending
    float *row_weight;      // [W][topk]
    int32_t *row_sel;       // [W][topk] top-k order
    int32_t *pair_slot;     // [W][topk] (problem*8 + row) of each selection's output
    int32_t *shared_slot;   // [W] the shared expert's output slot of each row
    int32_t *prob_rows;     // [pmax][8] source row of each problem row, -1: padding
    int32_t *prob_expert;   // [pmax] local weight slot of each problem
    int32_t *prob_count;    // [1]
    uint16_t *xg;           // [pmax][8][dim] gathered rows
    uint16_t *gu;           // [pmax][8][2*inter]
    uint16_t *yd;           // [pmax][8][dim]
};
int moe_rows_launch(const MoeDev &m, const MoeRows &w, const uint16_t *x, long ldx, int R, uint16_t *out, long ldo,
                    cudaStream_t st);

// x [R][ldx] BF16 device rows -> out [R][ldo] BF16.  forced: optional device
// [R][topk] selections replacing the computed top-k (the reference's
// teacher-forcing hook, c/gmoe.h:145-152).
int moe_forward_launch(const MoeDev &m, const uint16_t *x, long ldx, int R, uint16_t *out, long ldo,
                       const int32_t *forced, cudaStream_t st);
// The ordered combine alone (what moe_forward_launch with out == null leaves
// to the caller): out[r] = bf16 sum of the row's weighted expert outputs in
// ascending expert order, shared expert last.
int moe_combine_launch(const MoeDev &m, int R, uint16_t *out, long ldo, cudaStream_t st);

// Greedy picks over a vocabulary split across the expert-parallel group: one
// exchange publishes keys[0..R) (this rank's argmax keys), signals every
// peer, waits (bounded) for every peer's keys of the same exchange, and
// writes picks[r] = index of the largest key over all ranks (rows r >= n0,
// when n0 >= 0, go to picks2[r - n0] instead).
int ep_picks_exchange_launch(const EpCtx &ep, const unsigned long long *keys, int R, int *picks,
                             cudaStream_t st, int n0 = -1, int *picks2 = nullptr);
size_t ep_region_bytes(int dim);
// Every rank's vocabulary slice of logits rows [0, R) (written into the
// regions' logits areas by each rank's lm_head) gathered into logits
// [R][ldl] on this rank, then a barrier so that no rank writes its area
// again before every rank has read it.  Call after the lm_head's picks
// exchange (its barrier orders the writes before the reads).
int ep_logits_gather_launch(const EpCtx &ep, int R, uint16_t *logits, long ldl, cudaStream_t st);
// bytes of the prompt pass's part of a region (rows x topk contributions, two halves)
size_t ep_wide_bytes(int rows, int topk, int dim);
