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
GEN9BLAS_API int gen9blas_scal(int, int, double, void *, int) { G9_UNSUPPORTED("gen9blas_scal"); }
GEN9BLAS_API int gen9blas_copy(int, int, const void *, int, void *, int) { G9_UNSUPPORTED("gen9blas_copy"); }
GEN9BLAS_API int gen9blas_swap(int, int, void *, int, void *, int) { G9_UNSUPPORTED("gen9blas_swap"); }
GEN9BLAS_API int gen9blas_rot(int, int, void *, int, void *, int, double, double) { G9_UNSUPPORTED("gen9blas_rot"); }
GEN9BLAS_API int gen9blas_rotm(int, int, void *, int, void *, int, const double *) { G9_UNSUPPORTED("gen9blas_rotm"); }
GEN9BLAS_API void gen9blas_rotg(float *, float *, float *, float *) {
    fail(GEN9BLAS_ERR_UNSUPPORTED, "gen9blas_rotg is not part of the B200 hot path in this build");
}
GEN9BLAS_API void gen9blas_rotmg(float *, float *, float *, float, float *) {
    fail(GEN9BLAS_ERR_UNSUPPORTED, "gen9blas_rotmg is not part of the B200 hot path in this build");
}
GEN9BLAS_API int gen9blas_symv(int, int, int, double, const void *, int, const void *, int, double, void *, int) {
    G9_UNSUPPORTED("gen9blas_symv");
}
GEN9BLAS_API int gen9blas_trmv(int, int, int, int, int, const void *, int, void *, int) { G9_UNSUPPORTED("gen9blas_trmv"); }
GEN9BLAS_API int gen9blas_trsv(int, int, int, int, int, const void *, int, void *, int) { G9_UNSUPPORTED("gen9blas_trsv"); }
GEN9BLAS_API int gen9blas_syr(int, int, int, double, const void *, int, void *, int) { G9_UNSUPPORTED("gen9blas_syr"); }
GEN9BLAS_API int gen9blas_syr2(int, int, int, double, const void *, int, const void *, int, void *, int) {
    G9_UNSUPPORTED("gen9blas_syr2");
}
GEN9BLAS_API int gen9blas_gbmv(int, int, int, int, int, int, double, const void *, int, const void *, int, double, void *, int) {
    G9_UNSUPPORTED("gen9blas_gbmv");
}
GEN9BLAS_API int gen9blas_sbmv(int, int, int, int, double, const void *, int, const void *, int, double, void *, int) {
    G9_UNSUPPORTED("gen9blas_sbmv");
}
GEN9BLAS_API int gen9blas_tbmv(int, int, int, int, int, int, const void *, int, void *, int) { G9_UNSUPPORTED("gen9blas_tbmv"); }
GEN9BLAS_API int gen9blas_tbsv(int, int, int, int, int, int, const void *, int, void *, int) { G9_UNSUPPORTED("gen9blas_tbsv"); }
GEN9BLAS_API int gen9blas_spmv(int, int, int, double, const void *, const void *, int, double, void *, int) {
    G9_UNSUPPORTED("gen9blas_spmv");
}
GEN9BLAS_API int gen9blas_tpmv(int, int, int, int, int, const void *, void *, int) { G9_UNSUPPORTED("gen9blas_tpmv"); }
GEN9BLAS_API int gen9blas_tpsv(int, int, int, int, int, const void *, void *, int) { G9_UNSUPPORTED("gen9blas_tpsv"); }
GEN9BLAS_API int gen9blas_spr(int, int, int, double, const void *, int, void *) { G9_UNSUPPORTED("gen9blas_spr"); }
GEN9BLAS_API int gen9blas_spr2(int, int, int, double, const void *, int, const void *, int, void *) {
    G9_UNSUPPORTED("gen9blas_spr2");
}

}  // extern "C"
