// model_dev.h — device-side descriptors of the glm5_next decode stack
// (internal).  Every pointer is device memory.  R <= MAXR token rows per call.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "gmoe_dev.h"

#define MAXR 8            // rows of one forward (verify depth or prefill chunk)
#define NSLOT (MAXR + 1)  // KDA checkpoint ring: committed state + MAXR provisional

// Dimensions (field meaning of ApusGmodelConfig, c/gmodel.h:88-108).
struct Dims {
    int d, V, L, hc;
    float eps, hc_eps, lower_bound, route_scale, limit;
    int sinkhorn_iters;
    int H, D, Dr, K;                  // KDA: heads, head dim, low rank, conv width
    int qkv;                          // H*D
    int AH, qd, vd, ql, kl;           // DSA MLA
    int IH, ID, topk, kpool, tail;    // Lightning indexer
    int E, ktop, inter, dense_inter;  // MoE / dense MLP
};

// KDA projection rows (q|k|v|f_a|g_a|b) and the row stride of their
// scratch output, padded to 16 bytes so the low-rank f_b/g_b GEMV that reads
// f_a|g_a from it stays on the bulk-copy path.
inline int kda_nproj(const Dims &D) { return 3 * D.qkv + 2 * D.Dr + D.H; }
inline int kda_ldkp(const Dims &D) { return (kda_nproj(D) + 7) & ~7; }

// Control block of one sequence (device).  Positions are absolute.
struct Ctl {
    int pos;            // tokens committed to the main model
    int kda_cur;        // checkpoint slot holding the committed KDA state
    int mtp_n;          // tokens committed to the MTP block's caches
    int held;           // sampled, not yet emitted token (speculative mode)
    int matched;        // accepted drafts of the last step
    int drafts[MAXR];   // d1..dD
    int batch[MAXR];    // verify batch [held, d2..dD]
    int picks[MAXR];    // argmax of each verify row
    int emitted[MAXR + 1];
    int n_emitted;
    long long stat_emitted, stat_batches, stat_offered, stat_accepted;
    int err;            // sticky error (capacity)
    int log_n;          // tokens in the emitted-token log
    int chain_pos[MAXR];// MTP cache position of each draft-chain step
    int mtp_picks[MAXR];// argmax of each MTP row
    int one;            // constant 1 (row count of single-row launches)
    // forced draft agreement
    int force_on, force_base, force_n;
    unsigned long long force_seed;
    double force_p;
    // sampling (c/gmtp.h:208-209): temp <= 0 is greedy; rng_s is the
    // splitmix64 state, advanced once per sampled token
    float temp, top_p;
    unsigned long long rng_s;
    // the MTP's own drafts of the last chain, before any forced agreement
    int raw_drafts[MAXR];
    // ApusGspec counters the reference keeps beside the walk's (c/gmtp.h:
    // 786-787, 845): d1 = the first draft against the held token; refeed =
    // the tokens its partial-reject path re-decodes (the checkpoint ring
    // here re-decodes nothing; the count keeps the reference's meaning)
    long long stat_d1_hits, stat_d1_offered, stat_refeed, stat_batch_tokens;
};

struct KdaW {
    const uint16_t *proj;     // [3*qkv + 2*Dr + H][d]: q | k | v | f_a | g_a | b
    const uint16_t *fg_b;     // [2][qkv][Dr]: f_b | g_b
    const uint16_t *conv;     // [3*qkv][K]
    const float *A_log;       // [H]
    const float *dt_bias;     // [qkv]
    const uint16_t *o_norm;   // [D]
    const uint16_t *o_w;      // [d][qkv]
};

struct DsaW {
    const uint8_t *qkva_c;    // FP8 [ql + kl][d]: q_a | kv_a
    const float *qkva_s;      // [(ql+kl)/128][d/128]
    const uint16_t *q_a_norm, *kv_a_norm;
    const uint8_t *q_b_c;     // FP8 [AH*qd][ql]
    const float *q_b_s;
    const uint16_t *kv_b;     // BF16 [AH*(qd+vd)][kl]
    const uint8_t *o_c;       // FP8 [d][AH*vd]
    const float *o_s;
    const uint16_t *idx_wq_b; // BF16 [IH*ID][ql]
    const uint16_t *idx_kgw;  // BF16 [2*ID + IH][d]: wk | compress_gate | weights_proj
    const uint16_t *idx_knorm_w, *idx_knorm_b, *idx_ape;   // [ID], [ID], [kpool][ID]
};

struct LayerW {
    int is_dsa, sparse;
    const uint16_t *input_norm, *post_norm;
    const uint16_t *hc_fn[2];       // BF16 [(2+hc)*hc][hc*d]
    const float *hc_base[2], *hc_scale[2];
    KdaW kda;
    DsaW dsa;
    MoeDev moe;                     // sparse layers (and the dense MLP as expert 0)
};

struct KdaState {
    uint16_t *conv;   // [NSLOT][3*qkv][K-1]
    float *rec;       // [NSLOT][H][D][D]
};

struct DsaState {
    uint16_t *k, *v;  // [AH][cap][qd], [AH][cap][vd]
    uint16_t *ik, *ig;// [cap][ID] indexer key (LayerNorm'd) / compress gate
    uint16_t *pkey;   // [cap/kpool][ID] pool keys (BF16)
    int cap;
};

// Per-forward scratch (device), sized for MAXR rows.
struct Scratch {
    uint16_t *h4, *h4b;     // [R][hc*d] residual streams (ping-pong)
    uint16_t *x, *sub;      // [R][d]
    float *mix;             // [R][hc_nchunk][(2+hc)*hc + 1] pre-mix partials
    float *post, *comb;     // [R][hc], [R][hc*hc]
    uint16_t *kp;           // KDA projections [R][3qkv+2Dr+H]
    uint16_t *fgo;          // [2][R][qkv]  f_b, g_b outputs
    uint16_t *qkvc;         // [R][3qkv] post-conv
    uint16_t *core;         // [R][qkv] gated-normed core
    uint16_t *qkva, *qres, *kpass;  // [R][ql+kl], [R][ql], [R][kl]
    uint16_t *q;            // [R][AH*qd]
    uint16_t *kvb;          // [R][AH*(qd+vd)]
    uint16_t *iq;           // [R][IH*ID]
    uint16_t *ikgw;         // [R][2ID+IH]
    float *iscore;          // [R][maxpools]
    uint8_t *isel;          // [R][maxpools] pool selected
    uint16_t *attn;         // [R][AH*vd]
    float *attn_scores;     // [AH][MAXR][attn_sstride] attention scores
    uint16_t *attn_p;       // [AH][MAXR][attn_sstride] attention probabilities (BF16)
    int attn_sstride;       // >= cache capacity
    uint16_t *yn;           // [R][d] post-final-norm rows
    uint16_t *logits;       // [R][V] (optional)
    unsigned long long *amax;   // [R]
    int32_t *ids;           // [R] token ids of this forward
    // MTP glue
    uint16_t *eh;           // [R][2d]
    uint16_t *mx, *mxn;     // [R][d]
    uint16_t *oh;           // [R][d] post-shared_head.norm rows
    uint16_t *hprev;        // [R][d] hnorm inputs
    int *two_problems;      // {0, 1, 2}: the f_b / g_b problem list of one grouped GEMV and its count
    int maxpools;
};

// ---- layer kernels (layers.cu) -------------------------------------------
// Shape checks + kernel attributes for a model of dims D (once per model).
int layers_prepare(const Dims &D);
// All take the row count R and the device control block (positions).
int k_embed_launch(const uint16_t *embed, const int32_t *ids, int R, int d, int hc, uint16_t *h4,
                   cudaStream_t st);
// mHC of one site: the pre-mix partials in S.mix (left by hc_postmix_launch)
// -> S.x (the collapsed row normed with the input/post norm), S.post/comb.
int hc_pre_launch(const Dims &D, const LayerW &W, int site, const uint16_t *h4, int R, Scratch &S,
                  cudaStream_t st);
// The expand after a sublayer (h4out != null; the sublayer output is x [R][d],
// or, with x == null, the MoE outputs of *moe combined on the fly), then the
// pre-mix partials of the next site's fn_next (when given) into S.mix.  With
// h4out == null only the partials of the streams h4 are computed.
struct HcPostMix {
    const uint16_t *x;
    MoeDev moe;
    const uint16_t *h4;
    const float *post, *comb;
    uint16_t *h4out;
    const uint16_t *fn;
    float *part;                  // [R][nchunk][nmix + 1]
    int d, hc, nmix, R, nchunk;
};
int hc_nchunk(const Dims &D);
int hc_postmix_launch(const Dims &D, const uint16_t *x, const MoeDev *moe, const uint16_t *h4, int R, Scratch &S,
                      uint16_t *h4out, const uint16_t *fn_next, cudaStream_t st);
// The same over R rows of any count (MAXR rows a block row), the sublayer
// output always given as x rows.
int hc_postmix_rows_launch(const Dims &D, const uint16_t *x, const uint16_t *h4, int R, Scratch &S, uint16_t *h4out,
                           const uint16_t *fn_next, cudaStream_t st);
int head_norm_launch(const Dims &D, const uint16_t *h4, const uint16_t *norm_w, int R, uint16_t *yn,
                     unsigned long long *keys, cudaStream_t st);     // keys: zeroed for the lm_head argmax
int rmsnorm_rows_launch(const uint16_t *x, long ldx, const uint16_t *w, int n, int R, float eps,
                        uint16_t *y, long ldy, cudaStream_t st);
// One weighted RMSNorm per segment and row, up to 2 segments in one launch.
// Row r of a segment reads x + (gather ? gather[r] : r) * ldx; with sub, the
// row first becomes bf16(x + sub) and is written back to x (the residual add
// of c/gmtp.h:281-284).  keys (optional): zeroed for rows 0..R-1 (the argmax
// keys of the lm_head that follows).
struct NormSeg {
    const uint16_t *x; long ldx;
    const int32_t *gather;
    const uint16_t *sub; long ldsub;
    const uint16_t *w; int n;
    uint16_t *y; long ldy;
};
int norm_seg_launch(const NormSeg *seg, int nseg, int R, float eps, unsigned long long *keys, cudaStream_t st);
int kda_launch(const Dims &D, const LayerW &W, KdaState &KS, const Ctl *ctl, int R, Scratch &S,
               float *part, int *tick, cudaStream_t st);            // S.x -> S.sub
int dsa_launch(const Dims &D, const DsaW &W, DsaState &DS, const int *base_n, int R, Scratch &S,
               const uint16_t *x, uint16_t *out, float *part, int *tick, cudaStream_t st);
int residual_add_launch(uint16_t *x, const uint16_t *sub, long n, cudaStream_t st);
// Temperature / top-p draws of BF16 logits rows (c/sample.h:91-177): row r
// takes the (r+1)-th splitmix64 draw after the state *rng_dev (or rng_val
// when rng_dev is null) and writes its token to out[r]; temp <= 0 is the
// lowest-index argmax.  sample_prepare sets the kernel's shared-memory limit
// on the current device (before its first launch there, outside any stream
// capture).
int sample_prepare(int V);
int sample_launch(const uint16_t *logits, long ld, int V, int rows, float temp, float top_p,
                  const unsigned long long *rng_dev, unsigned long long rng_val, int *out, cudaStream_t st);

// ---- the prompt pass (prefill.cu; dsa_rows_launch in layers.cu) -----------
// Buffers of up to W prompt rows (device).  KDA, DSA and the dense MLP run one
// after another, so their row buffers share one arena.
struct KdaRows {
    int W;
    uint16_t *kp;           // [W][kda_ldkp]
    uint16_t *qkvc;         // [W][3qkv] post-conv
    uint16_t *fgo;          // [2][W][qkv] f_b, g_b outputs
    float *g;               // [W][qkv] forget gate (log decay)
    uint16_t *beta;         // [W][H]
    uint16_t *core;         // [W][qkv] chunked-core output
    uint16_t *onorm;        // [W][qkv] gated o_norm
};
struct DsaRows {
    uint16_t *qkva, *qres, *kpass, *q, *kvb, *iq, *ikgw, *attn;
    float *iscore;          // [W][maxpools]
    uint8_t *isel;          // [W][maxpools]
};
struct MlpRows {
    uint16_t *gu;           // [W][2*inter]
    uint16_t *h;            // [W][inter]
};
int iota_launch(int *a, int n, cudaStream_t st);
// The chunked KDA core (kda_chunk.cu) over s rows; q, k, v rows ldx elements
// apart (0: dense, H*D).
int kda_chunk_launch(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *g, const uint16_t *beta,
                     float *S, uint16_t *out, int s, int H, int D, cudaStream_t st, long ldx);
// The KDA sublayer over R <= X.W prompt rows x -> out, the conv window and the
// recurrent state taken from and left in the committed slot.
int kda_rows_launch(const Dims &D, const LayerW &W, uint16_t *conv_slot, float *rec_slot, int R, const KdaRows &X,
                    const uint16_t *x, uint16_t *out, cudaStream_t st);
// The DSA sublayer over R prompt rows at positions pos_iota[p0 ..] (pos_iota
// holds 0, 1, 2, ...): the chunk's K/V and indexer rows appended, then each
// row's indexer selection and attention over the positions <= its own.  FP8
// matrices are dequantised into wbuf for the GEMMs; attention runs in 8-row
// launches on S's attention scratch.
int dsa_rows_launch(const Dims &D, const DsaW &W, DsaState &DS, const int *pos_iota, int p0, int R,
                    const DsaRows &X, Scratch &S, uint16_t *wbuf, const uint16_t *x, uint16_t *out, cudaStream_t st);
int mlp_rows_launch(const MoeDev &md, int R, const MlpRows &X, uint16_t *wbuf, const uint16_t *x, uint16_t *out,
                    cudaStream_t st);
