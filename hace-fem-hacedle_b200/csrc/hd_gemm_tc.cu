// hd_gemm_tc.cu -- prefill Q-GEMM on the tcgen05 tensor cores (placeholder
// until the kernel lands; reports HD_E_UNSUPPORTED).
#include "hd_internal.cuh"

int hd_qgemm_tc(hd_ctx *ctx, const hd_weight *w, const float *X, float *Y, int T) {
    (void)w; (void)X; (void)Y; (void)T;
    return hd_fail(ctx, HD_E_UNSUPPORTED, "hd_qgemm: HD_PREC_BF16_TC not built yet");
}
