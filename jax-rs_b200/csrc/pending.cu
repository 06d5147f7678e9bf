// pending.cu -- entry points declared in include/jaxrs_cuda.h whose kernels
// are not in this build yet.  Each returns JX_EUNSUPPORTED with a message, so
// a caller fails loudly instead of silently computing nothing.
#include "jx_common.cuh"

#define JX_PENDING(name) return jx::fail(JX_EUNSUPPORTED, name ": not available in this build")

extern "C" {
int jx_fft_c2c_f32(const float*, float*, int64_t, int64_t, int, jx_stream_t) { JX_PENDING("jx_fft_c2c_f32"); }
int jx_fft2_c2c_f32(const float*, float*, int64_t, int64_t, int64_t, int, jx_stream_t) { JX_PENDING("jx_fft2_c2c_f32"); }
int jx_conv2d_fwd_f32(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                      int64_t, int64_t, int64_t, jx_stream_t) { JX_PENDING("jx_conv2d_fwd_f32"); }
int jx_conv2d_bwd_data_f32(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t, int64_t,
                           int64_t, int64_t, int64_t, int64_t, jx_stream_t) { JX_PENDING("jx_conv2d_bwd_data_f32"); }
int jx_conv2d_bwd_filter_f32(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t, int64_t,
                             int64_t, int64_t, int64_t, int64_t, jx_stream_t) { JX_PENDING("jx_conv2d_bwd_filter_f32"); }
int jx_softmax_rows_f32(const float*, float*, int64_t, int64_t, jx_stream_t) { JX_PENDING("jx_softmax_rows_f32"); }
int jx_softmax_xent_f32(const float*, const float*, float*, float*, float*, int64_t, int64_t, jx_stream_t) {
  JX_PENDING("jx_softmax_xent_f32");
}
int jx_bias_act_f32(float*, const float*, float*, int64_t, int64_t, int, jx_stream_t) { JX_PENDING("jx_bias_act_f32"); }
int jx_act_bwd_f32(const float*, const float*, float*, float*, int64_t, int64_t, int, jx_stream_t) {
  JX_PENDING("jx_act_bwd_f32");
}
int jx_col_sum_f32(const float*, float*, int64_t, int64_t, jx_stream_t) { JX_PENDING("jx_col_sum_f32"); }
int jx_adam_step_f32(float* const*, const float* const*, float* const*, float* const*, const int64_t*, int, float,
                     float, float, float, int64_t, jx_stream_t) { JX_PENDING("jx_adam_step_f32"); }
int jx_nccl_unique_id_size(void) { return 0; }
int jx_nccl_get_unique_id(void*) { JX_PENDING("jx_nccl_get_unique_id"); }
int jx_nccl_init(const void*, int, int, int, void**) { JX_PENDING("jx_nccl_init"); }
int jx_nccl_allreduce_sum_f32(void*, float*, int64_t, jx_stream_t) { JX_PENDING("jx_nccl_allreduce_sum_f32"); }
int jx_nccl_wait(void*, jx_stream_t, int) { JX_PENDING("jx_nccl_wait"); }
int jx_nccl_destroy(void*) { JX_PENDING("jx_nccl_destroy"); }
}
