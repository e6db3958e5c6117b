/* ref_stubs.c -- TEST INFRASTRUCTURE ONLY. Link-time stand-ins for the GPU entry points that the reference's CBLAS
 * layer (lib/src/cblas.c of kprzybys/gen9-gpu-blas) references, so that the layer builds as a pure CPU library:
 * gen9blas_init() reports "no device", which puts the layer into its CPU mode (cblas.c:66-78), and every call then
 * goes to the OpenBLAS named by GEN9BLAS_BLAS_CPU. None of the other stand-ins is ever reached in that mode; they
 * return the generic error code. Used only by oracle/Makefile to build oracle/_ref/libgen9blas_blas_ref.so. */
const char *gen9blas_error(void) { return "reference GPU path unavailable (Intel Gen9 iGPU required): CPU oracle build"; }
int gen9blas_init(void) { return -5; }
#define STUB(name) int name(void) { return -1; }
STUB(gen9blas_asum) STUB(gen9blas_axpy) STUB(gen9blas_copy) STUB(gen9blas_dot) STUB(gen9blas_gbmv) STUB(gen9blas_gemm)
STUB(gen9blas_gemv) STUB(gen9blas_ger) STUB(gen9blas_iamax) STUB(gen9blas_nrm2) STUB(gen9blas_rot) STUB(gen9blas_rotm)
STUB(gen9blas_sbmv) STUB(gen9blas_scal) STUB(gen9blas_spmv) STUB(gen9blas_spr) STUB(gen9blas_spr2) STUB(gen9blas_swap)
STUB(gen9blas_symm) STUB(gen9blas_symv) STUB(gen9blas_syr) STUB(gen9blas_syr2) STUB(gen9blas_syr2k) STUB(gen9blas_syrk)
STUB(gen9blas_tbmv) STUB(gen9blas_tbsv) STUB(gen9blas_tpmv) STUB(gen9blas_tpsv) STUB(gen9blas_trmm) STUB(gen9blas_trmv)
STUB(gen9blas_trsm) STUB(gen9blas_trsv)
