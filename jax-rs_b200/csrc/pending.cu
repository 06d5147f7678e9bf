// pending.cu -- entry points declared in include/jaxrs_cuda.h whose kernels
// are not in this build yet.  Each returns JX_EUNSUPPORTED with a message, so
// a caller fails loudly instead of silently computing nothing.
#include "jx_common.cuh"

#define JX_PENDING(name) return jx::fail(JX_EUNSUPPORTED, name ": not available in this build")

extern "C" {
int jx_conv2d_fwd_f32(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                      int64_t, int64_t, int64_t, jx_stream_t) { JX_PENDING("jx_conv2d_fwd_f32"); }
int jx_conv2d_bwd_data_f32(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t, int64_t,
                           int64_t, int64_t, int64_t, int64_t, jx_stream_t) { JX_PENDING("jx_conv2d_bwd_data_f32"); }
int jx_conv2d_bwd_filter_f32(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t, int64_t,
                             int64_t, int64_t, int64_t, int64_t, jx_stream_t) { JX_PENDING("jx_conv2d_bwd_filter_f32"); }
}
