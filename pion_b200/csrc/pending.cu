// Entry points whose kernels are not in this build yet: each reports ESHAPE with a
// message instead of computing anything.
#include <cstdio>

#include "internal.h"

using namespace pion;

extern "C" {

static int pending(pion_b200_ctx* ctx, const char* what) {
    if (ctx) set_error(ctx, PION_B200_ESHAPE, "%s: not available in this build", what);
    else fprintf(stderr, "pion_vector_b200: %s not available in this build\n", what);
    return PION_B200_ESHAPE;
}

int pion_v_b200_register_bq(pion_b200_ctx* ctx, const float*, int64_t, int64_t, int64_t, int, int,
                            pion_b200_index**) {
    return pending(ctx, "register_bq");
}
int pion_v_b200_bq_rerank_knn(pion_b200_ctx* ctx, const pion_b200_index*, const float*, int64_t,
                              int64_t, int64_t, int32_t*, float*, int) {
    return pending(ctx, "bq_rerank_knn");
}

}  // extern "C"
