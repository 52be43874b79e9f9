// onednn_flash_attention_op.cc -- the OneDNNFlashAttention TensorFlow op on the B200 kernel.
//
// Drop-in for the reference's tensorflow_ops/onednn_flash_attention_op.cc: the same op
// name, inputs, attributes, shape function and validation (lines 13-38 and 63-101 there),
// with
//   * a type attribute T in {float, bfloat16} that defaults to float, so graphs built
//     against the reference keep their signature;
//   * a DEVICE_GPU kernel that runs the sm_100a forward on TensorFlow's CUDA stream
//     through the C ABI (include/odf_sm100.h): fp32 inputs are converted to bf16 into
//     temporaries from TensorFlow's allocator, bf16 inputs are used in place;
//   * the DEVICE_CPU kernel kept: it runs the same forward through the host entry
//     (host buffers streamed through the current GPU).
// As in the reference, scale = 1/sqrt(D) and the attributes use_onednn / tile_kernel /
// qk_tile_layout are validated and otherwise ignored; query/key block sizes are validated
// (> 0) but the GPU tiles are 128 x 128.
//
// Build (needs TensorFlow headers; CUDA path with -DGOOGLE_CUDA=1):
//   TF_CFLAGS=$(python -c 'import tensorflow as tf; print(" ".join(tf.sysconfig.get_compile_flags()))')
//   TF_LFLAGS=$(python -c 'import tensorflow as tf; print(" ".join(tf.sysconfig.get_link_flags()))')
//   g++ -std=c++17 -shared -fPIC -O2 -DGOOGLE_CUDA=1 $TF_CFLAGS -I<repo>/include \
//       onednn_flash_attention_op.cc -o onednn_flash_tf_attention.so \
//       -L<repo>/dnn-flash_b200/lib -lodf_sm100 $TF_LFLAGS -Wl,-rpath,<repo>/dnn-flash_b200/lib
#include <cmath>
#include <cstring>
#include <string>
#include <type_traits>

#include "odf_sm100.h"
#include "tensorflow/core/framework/op.h"
#include "tensorflow/core/framework/op_kernel.h"
#include "tensorflow/core/framework/shape_inference.h"

#if GOOGLE_CUDA
#define EIGEN_USE_GPU
#include "tensorflow/core/util/gpu_kernel_helper.h"
#endif

using namespace tensorflow;  // NOLINT

REGISTER_OP("OneDNNFlashAttention")
    .Input("q: T")
    .Input("k: T")
    .Input("v: T")
    .Output("out: float")
    .Attr("T: {float, bfloat16} = DT_FLOAT")
    .Attr("causal: bool = true")
    .Attr("query_block_size: int = 16")
    .Attr("key_block_size: int = 32")
    .Attr("use_onednn: bool = true")
    .Attr("tile_kernel: string = 'onednn'")
    .Attr("qk_tile_layout: string = 'strided_k'")
    .SetShapeFn([](shape_inference::InferenceContext* c) {
        shape_inference::ShapeHandle q, k, v;
        TF_RETURN_IF_ERROR(c->WithRank(c->input(0), 4, &q));
        TF_RETURN_IF_ERROR(c->WithRank(c->input(1), 4, &k));
        TF_RETURN_IF_ERROR(c->WithRank(c->input(2), 4, &v));
        c->set_output(0, c->MakeShape({c->Dim(q, 0), c->Dim(q, 1), c->Dim(q, 2), c->Dim(v, 3)}));
        return OkStatus();
    });

namespace {

// Attribute and shape checks shared by both device kernels (reference op.cc:58-101).
class FlashAttentionBase : public OpKernel {
public:
    explicit FlashAttentionBase(OpKernelConstruction* ctx) : OpKernel(ctx) {
        OP_REQUIRES_OK(ctx, ctx->GetAttr("causal", &causal_));
        OP_REQUIRES_OK(ctx, ctx->GetAttr("query_block_size", &query_block_size_));
        OP_REQUIRES_OK(ctx, ctx->GetAttr("key_block_size", &key_block_size_));
        std::string tile_kernel, layout;
        OP_REQUIRES_OK(ctx, ctx->GetAttr("tile_kernel", &tile_kernel));
        OP_REQUIRES_OK(ctx, ctx->GetAttr("qk_tile_layout", &layout));
        OP_REQUIRES(ctx, tile_kernel == "onednn" || tile_kernel == "onednn_brgemm",
                    errors::InvalidArgument("tile_kernel must be 'onednn' or 'onednn_brgemm'"));
        OP_REQUIRES(ctx, layout == "strided_k" || layout == "copied_transposed" || layout == "brgemm_transformed_k",
                    errors::InvalidArgument(
                        "qk_tile_layout must be 'strided_k', 'copied_transposed', or 'brgemm_transformed_k'"));
    }

protected:
    // Validates inputs, allocates the output and fills the shape part of `p`; on failure
    // the context carries the error (callers check ctx->status()).
    void Prepare(OpKernelContext* ctx, odf_fwd_params* p, Tensor** out) {
        const Tensor& q = ctx->input(0);
        const Tensor& k = ctx->input(1);
        const Tensor& v = ctx->input(2);
        OP_REQUIRES(ctx, q.dims() == 4, errors::InvalidArgument("q must be rank 4 [B,H,M,D]"));
        OP_REQUIRES(ctx, k.dims() == 4, errors::InvalidArgument("k must be rank 4 [B,H,N,D]"));
        OP_REQUIRES(ctx, v.dims() == 4, errors::InvalidArgument("v must be rank 4 [B,H,N,Dv]"));
        OP_REQUIRES(ctx, q.dim_size(0) == k.dim_size(0) && q.dim_size(0) == v.dim_size(0),
                    errors::InvalidArgument("batch dimensions must match"));
        OP_REQUIRES(ctx, q.dim_size(1) % k.dim_size(1) == 0 && k.dim_size(1) == v.dim_size(1),
                    errors::InvalidArgument("head dimensions must match (q heads a multiple of k/v heads)"));
        OP_REQUIRES(ctx, q.dim_size(3) == k.dim_size(3), errors::InvalidArgument("q/k head dimensions must match"));
        OP_REQUIRES(ctx, k.dim_size(2) == v.dim_size(2),
                    errors::InvalidArgument("k/v key-token dimensions must match"));
        OP_REQUIRES(ctx, query_block_size_ > 0 && key_block_size_ > 0,
                    errors::InvalidArgument("block sizes must be positive"));
        TensorShape out_shape({q.dim_size(0), q.dim_size(1), q.dim_size(2), v.dim_size(3)});
        OP_REQUIRES_OK(ctx, ctx->allocate_output(0, out_shape, out));
        std::memset(p, 0, sizeof(*p));
        p->batch = q.dim_size(0);
        p->heads_q = q.dim_size(1);
        p->heads_kv = k.dim_size(1);
        p->seqlen_q = q.dim_size(2);
        p->seqlen_k = k.dim_size(2);
        p->head_dim = q.dim_size(3);
        p->value_dim = v.dim_size(3);
        p->scale = 1.0f / std::sqrt(static_cast<float>(p->head_dim));
        p->causal = causal_ ? 1 : 0;
        p->o_dtype = ODF_DTYPE_F32;
        p->o = (*out)->flat<float>().data();
    }

    static Status ToStatus(int rc, const char* what) {
        if (rc == ODF_OK) return OkStatus();
        const std::string msg = std::string(what) + ": " + odf_last_error();
        if (rc == ODF_ERR_INVALID_ARG) return errors::InvalidArgument(msg);
        return errors::Internal("OneDNNFlashAttention failed: ", msg);
    }

    bool causal_ = true;
    int query_block_size_ = 16;
    int key_block_size_ = 32;
};

// Host tensors: the host entry streams them through the current GPU.
template <typename T>
class FlashAttentionCpuOp final : public FlashAttentionBase {
public:
    using FlashAttentionBase::FlashAttentionBase;
    void Compute(OpKernelContext* ctx) override {
        odf_fwd_params p;
        Tensor* out = nullptr;
        Prepare(ctx, &p, &out);
        if (!ctx->status().ok()) return;
        p.q = ctx->input(0).tensor_data().data();
        p.k = ctx->input(1).tensor_data().data();
        p.v = ctx->input(2).tensor_data().data();
        p.qkv_dtype = std::is_same<T, float>::value ? ODF_DTYPE_F32 : ODF_DTYPE_BF16;
        OP_REQUIRES_OK(ctx, ToStatus(odf_flash_fwd_host(&p), "host entry"));
    }
};

REGISTER_KERNEL_BUILDER(Name("OneDNNFlashAttention").Device(DEVICE_CPU).TypeConstraint<float>("T"),
                        FlashAttentionCpuOp<float>);
REGISTER_KERNEL_BUILDER(Name("OneDNNFlashAttention").Device(DEVICE_CPU).TypeConstraint<bfloat16>("T"),
                        FlashAttentionCpuOp<bfloat16>);

#if GOOGLE_CUDA
// Device tensors on TensorFlow's stream; fp32 inputs are staged as bf16 temporaries.
template <typename T>
class FlashAttentionGpuOp final : public FlashAttentionBase {
public:
    using FlashAttentionBase::FlashAttentionBase;
    void Compute(OpKernelContext* ctx) override {
        odf_fwd_params p;
        Tensor* out = nullptr;
        Prepare(ctx, &p, &out);
        if (!ctx->status().ok()) return;
        void* stream = ctx->eigen_device<Eigen::GpuDevice>().stream();
        const Tensor* in[3] = {&ctx->input(0), &ctx->input(1), &ctx->input(2)};
        Tensor staged[3];
        const void* ptr[3];
        for (int i = 0; i < 3; ++i) {
            if (std::is_same<T, float>::value) {
                OP_REQUIRES_OK(ctx, ctx->allocate_temp(DT_BFLOAT16, in[i]->shape(), &staged[i]));
                OP_REQUIRES_OK(ctx, ToStatus(odf_convert_f32_to_bf16(
                                                 reinterpret_cast<const float*>(in[i]->tensor_data().data()),
                                                 reinterpret_cast<uint16_t*>(const_cast<char*>(
                                                     staged[i].tensor_data().data())),
                                                 in[i]->NumElements(), stream),
                                             "fp32 -> bf16 staging"));
                ptr[i] = staged[i].tensor_data().data();
            } else {
                ptr[i] = in[i]->tensor_data().data();
            }
        }
        p.q = ptr[0];
        p.k = ptr[1];
        p.v = ptr[2];
        p.qkv_dtype = ODF_DTYPE_BF16;
        // workspace: the kernel's work-item counter (TensorFlow's allocator, 64-byte aligned)
        Tensor ws;
        const size_t wbytes = odf_fwd_workspace_size(&p);
        OP_REQUIRES_OK(ctx, ctx->allocate_temp(DT_INT8, TensorShape({static_cast<int64_t>(wbytes)}), &ws));
        p.workspace = const_cast<char*>(ws.tensor_data().data());
        p.workspace_bytes = wbytes;
        OP_REQUIRES_OK(ctx, ToStatus(odf_flash_fwd_sm100(&p, stream), "device entry"));
    }
};

REGISTER_KERNEL_BUILDER(Name("OneDNNFlashAttention").Device(DEVICE_GPU).TypeConstraint<float>("T"),
                        FlashAttentionGpuOp<float>);
REGISTER_KERNEL_BUILDER(Name("OneDNNFlashAttention").Device(DEVICE_GPU).TypeConstraint<bfloat16>("T"),
                        FlashAttentionGpuOp<bfloat16>);
#endif  // GOOGLE_CUDA

}  // namespace
