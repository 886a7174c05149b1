// Decode GEMV with two CTAs per SM (8 consumer warps each, about half the
// shared memory each): one CTA's prologue (activation staging, outlier and
// bias table) overlaps the other CTA's streaming. Used when its shared-memory
// plan holds every token of the call in one pass and the caller's workspace
// covers its larger partial-sum area (twice the CTAs); otherwise the
// one-CTA-per-SM build of the same source runs.
#define TS_GEMV_NS gemv_v2
#define TS_GEMV_CW 8
#define TS_GEMV_CPS 2
// 512 outliers preloaded per CTA (more are read in place) so that the
// activations of a 14336-column down projection fit half an SM
#define TS_GEMV_OUTCAP 512
#include "qgemv.cu"
