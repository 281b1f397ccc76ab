/*
 * ref_glue.c — instantiates the apus reference's own header-only C engine
 * (c/*.h, compiled where it lies, never copied) into oracle/_ref/libapus_ref.so
 * so the tests can pin the oracle restatement against the reference itself
 * and the bench can time the reference CPU path.  TEST INFRASTRUCTURE ONLY.
 * The single-TU instantiation list mirrors tests/m8g/test_m8g.c:48-60.
 */
#define APUS_JSON_IMPLEMENTATION
#define APUS_ST_IMPLEMENTATION
#define APUS_COMPAT_IMPLEMENTATION
#define APUS_BF16_IMPLEMENTATION
#define APUS_FP8BLK_IMPLEMENTATION
#define APUS_GMHC_IMPLEMENTATION
#define APUS_GMOE_IMPLEMENTATION
#define APUS_GKDA_IMPLEMENTATION
#define APUS_GDSA_IMPLEMENTATION
#define APUS_GCACHE_IMPLEMENTATION
#define APUS_GMODEL_IMPLEMENTATION
#define APUS_SAMPLE_IMPLEMENTATION
#define APUS_GMTP_IMPLEMENTATION
#include "gmodel.h"
#include "gmtp.h"
#include "sample.h"
#include "bf16.h"
#include "fp8blk.h"

/* thread count the reference pool will use (c/pool.h APUS_THREADS) */
int apus_ref_threads(void) { return apus_pool_default_threads(); }
