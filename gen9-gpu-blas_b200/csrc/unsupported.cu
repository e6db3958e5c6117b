// unsupported.cu -- entry points of gen9blas.h that lie outside the hot path of this build (level-3 derived
// operations, constant packed weights, the rest of levels 1-2, banded and packed matrices). They stay exported so
// that the ABI is complete and programs linking any reference symbol still load; each returns
// GEN9BLAS_ERR_UNSUPPORTED (NULL for pack_b) with an explanatory error text.
#include "internal.h"

using namespace g9;

#define G9_UNSUPPORTED(name)                                                                         \
    do {                                                                                             \
        if (int e_ = begin_op()) return e_;                                                          \
        return fail(GEN9BLAS_ERR_UNSUPPORTED, "%s is not part of the B200 hot path in this build", name); \
    } while (0)

extern "C" {

GEN9BLAS_API gen9blas_packed_b *gen9blas_pack_b(int, int, int, int, const void *, int) {
    if (begin_op()) return nullptr;
    fail(GEN9BLAS_ERR_UNSUPPORTED, "gen9blas_pack_b is not part of the B200 hot path in this build");
    return nullptr;
}
GEN9BLAS_API int gen9blas_gemm_pb(int, int, double, const void *, int, const gen9blas_packed_b *, double, void *, int) {
    G9_UNSUPPORTED("gen9blas_gemm_pb");
}
GEN9BLAS_API void gen9blas_packed_b_free(gen9blas_packed_b *) {}

}  // extern "C"
