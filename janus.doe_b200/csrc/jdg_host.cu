// jdg_host.cu — host GGUF model half of the engine (placeholder until the packed kernels land).
#include "jdg_engine.h"

int jdg_enqueue_host_step(jdg_engine *e, int B) { (void)e; (void)B; return JD_EUNSUPPORTED; }
int jdg_host_set_attrs(jdg_engine *e) { (void)e; return JD_OK; }
void jdg_host_release(jdg_engine *e) { (void)e; }
extern "C" int jdg_host_upload(jdg_ctx *ctx, const jd_host_model *h, int max_batch, int max_seq, jdg_engine **out) {
    (void)ctx; (void)h; (void)max_batch; (void)max_seq; (void)out; return JD_EUNSUPPORTED;
}
extern "C" int jdg_comm_unique_id(void *id) { (void)id; return JD_EUNSUPPORTED; }
extern "C" int jdg_host_upload_tp(jdg_ctx *ctx, const jd_host_model *h, int max_batch, int max_seq, int rank, int world,
                                  const void *id, jdg_engine **out) {
    (void)ctx; (void)h; (void)max_batch; (void)max_seq; (void)rank; (void)world; (void)id; (void)out;
    return JD_EUNSUPPORTED;
}
extern "C" int jdg_qmatvec(jdg_ctx *ctx, float *out, const void *W, int dt, const float *x, int r, int c, int B) {
    (void)ctx; (void)out; (void)W; (void)dt; (void)x; (void)r; (void)c; (void)B; return JD_EUNSUPPORTED;
}
