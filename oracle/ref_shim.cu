// C-ABI shim over the REFERENCE kernels of comfyui-turing-utils (TEST
// INFRASTRUCTURE ONLY).  oracle/Makefile compiles this file together with the
// reference's own sources, read in place from the reference tree
// (kernel/csrc/turing/{convrot_quant,bf16_epilogue,w4a8}.cu), into
// oracle/_ref/libctu_ref.so.  Only tests/golden/make_golden.py and the tests
// load it, to pin the CPU oracle against the reference's device results.
//
// Each entry builds the reference's ATen-free `Tensor` views
// (kernel/csrc/tensor_bridge.h:137-236) over caller pointers, pushes the caller's
// stream on the reference's thread-local stream stack (tensor_bridge.h:57-61,
// as bindings.cpp:17-31 does) and calls the reference host entry.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <exception>
#include <string>

#include "kernel_api.h"

namespace ref = comfyui_turing_utils::kernels;

namespace {

thread_local std::string g_last_error;

Tensor view(void *ptr, std::initializer_list<int> shape, Tensor::ScalarType type) {
    Tensor t;
    t.ptr = ptr;
    t.scalarType = type;
    for (int d : shape) t.shape.dataExtent.push_back(d);
    int device = 0;
    cudaGetDevice(&device);
    t.dev = Device{Device::CUDA, device};
    return t;
}

struct StreamScope {
    explicit StreamScope(void *stream) { stackCUDAStreams.push_back(static_cast<cudaStream_t>(stream)); }
    ~StreamScope() { stackCUDAStreams.pop_back(); }
};

template <typename F>
int guarded(F &&fn) {
    try {
        fn();
        return 0;
    } catch (const std::exception &e) {
        g_last_error = e.what();
        return 1;
    }
}

}  // namespace

extern "C" {

const char *ref_last_error() { return g_last_error.c_str(); }

// kernel/csrc/turing/convrot_quant.cu:665-713 (row-buffer int8 / int4, optional SwiGLU).
int ref_bf16_convrot_quantize(const void *x, void *codes, void *scales, int rows, int k,
                              int bits, int swiglu, int block_threads, void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        const int width = swiglu ? 2 * k : k;
        Tensor in = view(const_cast<void *>(x), {rows, width}, Tensor::BF16);
        Tensor out = view(codes, {rows, bits == 4 ? k / 2 : k}, Tensor::INT8);
        Tensor sc = view(scales, {rows, 1}, Tensor::FP32);
        if (bits == 4) {
            ref::turing_bf16_int4_convrot_quantize(in, out, sc, swiglu != 0, block_threads);
        } else {
            ref::turing_bf16_int8_convrot_quantize(in, out, sc, swiglu != 0, block_threads);
        }
    });
}

// kernel/csrc/turing/convrot_quant.cu:715-745 (row-buffer tanh-GELU int8 / int4).
int ref_bf16_gelu_convrot_quantize(const void *x, void *codes, void *scales, int rows, int k,
                                   int bits, int block_threads, void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        Tensor in = view(const_cast<void *>(x), {rows, k}, Tensor::BF16);
        Tensor out = view(codes, {rows, bits == 4 ? k / 2 : k}, Tensor::INT8);
        Tensor sc = view(scales, {rows, 1}, Tensor::FP32);
        if (bits == 4) {
            ref::turing_bf16_gelu_int4_convrot_quantize(in, out, sc, block_threads);
        } else {
            ref::turing_bf16_gelu_int8_convrot_quantize(in, out, sc, block_threads);
        }
    });
}

// kernel/csrc/turing/w4a8.cu:1185-1219 (W8A8 GEMM + dequant/bias epilogue).
int ref_int8_linear(const void *a, const void *w, const void *a_scale, const void *w_scale,
                    const void *bias, void *out, int m, int n, int k, int tile_policy, void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        ref::turing_int8_linear(view(const_cast<void *>(a), {m, k}, Tensor::INT8),
                                view(const_cast<void *>(w), {n, k}, Tensor::INT8),
                                view(const_cast<void *>(a_scale), {m}, Tensor::FP32),
                                view(const_cast<void *>(w_scale), {n}, Tensor::FP32),
                                bias ? view(const_cast<void *>(bias), {n}, Tensor::FP32) : Tensor{},
                                view(out, {m, n}, Tensor::BF16), tile_policy);
    });
}

// kernel/csrc/turing/w4a8.cu:1000-1086 (signed packed-int4 W4A8, N % 8 == 0).
int ref_w4a8_linear(const void *a, const void *w_packed, const void *a_scale, const void *w_scale,
                    const void *bias, void *out, int m, int n, int k, int tile_policy, void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        ref::turing_w4a8_linear(view(const_cast<void *>(a), {m, k}, Tensor::INT8),
                                view(const_cast<void *>(w_packed), {n, k / 2}, Tensor::INT8),
                                view(const_cast<void *>(a_scale), {m}, Tensor::FP32),
                                view(const_cast<void *>(w_scale), {n}, Tensor::FP32),
                                bias ? view(const_cast<void *>(bias), {n}, Tensor::FP32) : Tensor{},
                                view(out, {m, n}, Tensor::BF16), tile_policy);
    });
}

// kernel/csrc/turing/bf16_epilogue.cu:146-217 (int32 accumulator -> bf16).
int ref_dequantize_int8_bf16(const void *acc, const void *a_scale, const void *w_scale,
                             int w_scale_count, void *out, int m, int acc_cols, int out_cols,
                             void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        Tensor accumulator = view(const_cast<void *>(acc), {m, acc_cols}, Tensor::INT32);
        ref::turing_dequantize_int8_bf16(accumulator,
                                         view(const_cast<void *>(a_scale), {m}, Tensor::FP32),
                                         view(const_cast<void *>(w_scale), {w_scale_count}, Tensor::FP32),
                                         view(out, {m, out_cols}, Tensor::BF16));
    });
}

// kernel/csrc/turing/w4a8.cu:1088-1182 (grouped-codebook W4A8: per-chunk decode to an
// int8 workspace + W8A8 GEMM, or the inline-decode CUTLASS iterator when
// inline_decode != 0, which needs group_size 16).
int ref_codebook_w4a8_linear(const void *a, const void *w_packed, const void *a_scale, const void *group_scale,
                             const void *channel_scale, const void *codebook, const void *bias, void *workspace,
                             int workspace_rows, void *out, int m, int n, int k, int group_size, int inline_decode,
                             int tile_policy, void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        ref::turing_codebook_w4a8_linear(
            view(const_cast<void *>(a), {m, k}, Tensor::INT8),
            view(const_cast<void *>(w_packed), {n, k / 2}, Tensor::INT8),
            view(const_cast<void *>(a_scale), {m}, Tensor::FP32),
            view(const_cast<void *>(group_scale), {n, k / group_size}, Tensor::FP8_E4M3),
            view(const_cast<void *>(channel_scale), {n}, Tensor::FP32),
            view(const_cast<void *>(codebook), {16}, Tensor::FP32),
            bias ? view(const_cast<void *>(bias), {n}, Tensor::FP32) : Tensor{},
            workspace ? view(workspace, {workspace_rows, k}, Tensor::INT8) : Tensor{},
            view(out, {m, n}, Tensor::BF16), group_size, inline_decode != 0, tile_policy);
    });
}

// kernel/csrc/turing/convrot_quant.cu:591-621 (SwiGLU shard with given row scales).
int ref_swiglu_int8_convrot_quantize_scaled(const void *x, const void *scales, void *codes, int rows, int k,
                                            void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        ref::turing_swiglu_int8_convrot_quantize_scaled(view(const_cast<void *>(x), {rows, 2 * k}, Tensor::BF16),
                                                        view(const_cast<void *>(scales), {rows}, Tensor::FP32),
                                                        view(codes, {rows, k}, Tensor::INT8));
    });
}

// The same on fp16 rows.
int ref_swiglu_int8_convrot_quantize_scaled_f16(const void *x, const void *scales, void *codes, int rows, int k,
                                                void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        ref::turing_swiglu_int8_convrot_quantize_scaled(view(const_cast<void *>(x), {rows, 2 * k}, Tensor::FP16),
                                                        view(const_cast<void *>(scales), {rows}, Tensor::FP32),
                                                        view(codes, {rows, k}, Tensor::INT8));
    });
}

// kernel/csrc/turing/convrot_quant.cu:535-663 (the staged two-kernel quantizers: rotate +
// per-group absmax into `rotated` / `partial`, then quantize from the partials).
// act 1 = SwiGLU (x is [rows, 2k]), 2 = tanh-GELU; bf16 input, or fp16 when fp16 != 0.
int ref_staged_convrot_quantize(const void *x, void *codes, void *scales, void *rotated, void *partial, int rows,
                                int k, int bits, int act, int fp16, void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        const Tensor::ScalarType t = fp16 ? Tensor::FP16 : Tensor::BF16;
        Tensor in = view(const_cast<void *>(x), {rows, act == 1 ? 2 * k : k}, t);
        Tensor rot = view(rotated, {rows, k}, t);
        Tensor part = view(partial, {rows, k / 256}, Tensor::FP32);
        Tensor out = view(codes, {rows, bits == 4 ? k / 2 : k}, Tensor::INT8);
        Tensor sc = view(scales, {rows, 1}, Tensor::FP32);
        if (act == 1) {
            if (bits == 4) ref::turing_swiglu_int4_convrot_quantize(in, rot, part, out, sc);
            else ref::turing_swiglu_int8_convrot_quantize(in, rot, part, out, sc);
        } else {
            if (bits == 4) ref::turing_gelu_int4_convrot_quantize(in, rot, part, out, sc);
            else ref::turing_gelu_int8_convrot_quantize(in, rot, part, out, sc);
        }
    });
}

namespace {
Tensor::ScalarType float_type(int dtype) {
    return dtype == 0 ? Tensor::BF16 : dtype == 1 ? Tensor::FP16 : Tensor::FP32;
}
}  // namespace

// kernel/csrc/turing/segmented_rms_adaln.cu:288-340 (affine RMSNorm + segmented AdaLN).
// dtype 0 = bf16, 1 = fp16, 2 = fp32; scale/shift rows are `*_stride` elements apart.
int ref_segmented_rms_adaln(const void *x, const void *weight, const void *scale, const void *shift,
                            const void *segments, void *out, int rows, int hidden, int param_rows,
                            int scale_stride, int shift_stride, int segment_count, float epsilon, int dtype,
                            void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        const Tensor::ScalarType t = float_type(dtype);
        Tensor sc = view(const_cast<void *>(scale), {param_rows, hidden}, t);
        sc.shape.dataStride = {scale_stride, 1};
        Tensor sh = view(const_cast<void *>(shift), {param_rows, hidden}, t);
        sh.shape.dataStride = {shift_stride, 1};
        ref::turing_segmented_rms_adaln(view(const_cast<void *>(x), {rows, hidden}, t),
                                        view(const_cast<void *>(weight), {hidden}, t), sc, sh,
                                        view(const_cast<void *>(segments), {segment_count, 3}, Tensor::INT32),
                                        view(out, {rows, hidden}, t), epsilon);
    });
}

// kernel/csrc/turing/segmented_rms_adaln.cu:365-407 (LayerNorm + Wan AdaLN).
int ref_layer_norm_adaln(const void *x, const void *scale, const void *shift, void *out, int batch, int sequence,
                         int hidden, int modulation_steps, float epsilon, int dtype, void *stream) {
    return guarded([&] {
        StreamScope scope(stream);
        const Tensor::ScalarType t = float_type(dtype);
        ref::turing_layer_norm_adaln(view(const_cast<void *>(x), {batch, sequence, hidden}, t),
                                     view(const_cast<void *>(scale), {batch, modulation_steps, hidden}, t),
                                     view(const_cast<void *>(shift), {batch, modulation_steps, hidden}, t),
                                     view(out, {batch, sequence, hidden}, t), epsilon);
    });
}

}  // extern "C"
