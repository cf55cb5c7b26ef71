/*
 * dcn_b200.h -- C ABI of the B200 (sm_100a) DCNv2 operator library (libdcn_b200.so).
 *
 * Modulated deformable convolution (DCNv2): for every output pixel p and kernel
 * tap t, the input is sampled bilinearly at the tap's position moved by a learned
 * offset, scaled by a learned mask, and the samples are contracted with the weight:
 *   y[b,co,p] = bias[co] + sum_{c,t} W[co,c,t] * mask[b,g(c)*T+t,p]
 *                                  * bilinear(x[b,c], pos(p,t) + offset[b,g(c),t,p])
 *
 * The entry points replace the reference operator's native layer one for one:
 *   dcn_forward  <- MyDCN_forward   (reference name.h:15-24, com.cu:198-272,
 *                                    bound as Conv2d._C.dcn_v2_forward, ext.cpp:16)
 *   dcn_backward <- MyDCN_backward  (reference name.h:26-36, com.cu:733-848,
 *                                    bound as Conv2d._C.dcn_v2_backward, ext.cpp:17)
 * Tensor arguments keep the reference's order (input, weight, mask, offset, bias[,
 * grad_output]) and its layouts: NCHW input, weight [Co][C][kh][kw], offset
 * [B][dg*2*kh*kw][Ho][Wo] with channel 2t = dh and 2t+1 = dw of tap t = i*kw + j,
 * mask [B][dg*kh*kw][Ho][Wo], output [B][Co][Ho][Wo].  All tensors are dense,
 * contiguous device memory of one element type.  Beyond the reference: dilation
 * and deformable groups are honoured, f16/bf16 tensors are accepted as well as
 * f32, and with desc.layout = DCN_NHWC every activation tensor (input, offset,
 * mask, output, grad_output and the gradients of input, offset and mask) is
 * channels-last instead ([B][H][W][C], [B][Ho][Wo][2*dg*kh*kw], ...), so stacked
 * layers pass activations on without layout passes.
 *
 * Calls are asynchronous on the given CUDA stream (NULL = legacy default stream);
 * nothing is allocated: the caller passes a device workspace of at least the
 * size reported by dcn_*_workspace_size.  Functions return DCN_OK or a negative
 * DCN_E* code and never throw.  Errors found on the device (a pipeline wait that
 * timed out) are OR-ed into an int in the workspace, readable with
 * dcn_read_device_status().
 */
#ifndef DCN_B200_H
#define DCN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DCN_API __attribute__((visibility("default")))
#else
#define DCN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element type of every tensor argument */
enum dcn_dtype { DCN_F32 = 0, DCN_F16 = 1, DCN_BF16 = 2 };

/* memory layout of the activation tensors (input, offset, mask, output and
 * their gradients); the weight is always [Co][C][kh][kw] */
enum dcn_layout {
  DCN_NCHW = 0, /* [B][C][H][W], the reference's layout */
  DCN_NHWC = 1  /* channels-last [B][H][W][C] (PyTorch channels_last memory format) */
};

/* return codes */
enum dcn_status_code {
  DCN_OK = 0,
  DCN_E_INVALID = -1,       /* bad shape / parameter */
  DCN_E_NULLPTR = -2,       /* a required pointer is NULL */
  DCN_E_WORKSPACE = -3,     /* workspace too small or misaligned */
  DCN_E_CUDA = -4,          /* a CUDA runtime call failed (launch error) */
  DCN_E_UNSUPPORTED = -5,   /* valid but unsupported configuration */
  DCN_E_DEVICE = -6,        /* error recorded by a kernel (see device status) */
  DCN_E_SCRATCH_LIMIT = -7  /* problem needs more scratch than dcn_forward_noalloc has */
};

/* device-side error bits (dcn_read_device_status) */
#define DCN_DEVERR_TIMEOUT 1 /* an mbarrier wait exceeded its limit; kernel gave up */

/* Problem description.  Output size: Ho = (H + 2*ph - (dh*(kh-1)+1))/sh + 1,
 * likewise Wo (reference com.cu:227-228 with dilation 1). */
typedef struct dcn_desc {
  int32_t B, C, H, W; /* input [B][C][H][W] */
  int32_t Co;         /* output channels */
  int32_t kh, kw;     /* kernel size */
  int32_t sh, sw;     /* stride */
  int32_t ph, pw;     /* zero padding */
  int32_t dh, dw;     /* dilation (reference: always 1) */
  int32_t dg;         /* deformable groups; C % dg == 0 (reference: always 1) */
  int32_t dtype;      /* enum dcn_dtype */
  int32_t has_bias;   /* 0: bias pointer ignored / grad_bias not written */
  int32_t layout;     /* enum dcn_layout; 0 (NCHW) in a zero-initialised descriptor */
  int32_t flags;      /* DCN_FLAG_* bits; 0 in a zero-initialised descriptor */
} dcn_desc;

/* dcn_desc.flags.  Both let a caller that keeps one workspace across calls skip
 * a packing pass whose result is already in it (no counterpart in the
 * reference, which re-derives everything per call).
 *
 * DCN_FLAG_INPUT_PACKED (dcn_backward, dcn_backward_om): `workspace` was passed,
 *   with the same descriptor and `input`, to the dcn_forward / dcn_forward_om
 *   call that this backward follows, and nothing has written to it since: the
 *   packed input it holds is reused instead of packing `input` again.  The
 *   workspace must then have dcn_backward_workspace_size bytes for both calls
 *   (the two layouts share the packed-input region).
 * DCN_FLAG_WEIGHT_PACKED (dcn_forward, dcn_forward_om): `workspace` holds the
 *   packed weight of an earlier forward call with the same descriptor and the
 *   same `weight` contents: the weight pack is skipped.
 * dcn_forward_noalloc ignores both flags. */
#define DCN_FLAG_INPUT_PACKED 1
#define DCN_FLAG_WEIGHT_PACKED 2

/* Validates `d` and writes the output spatial size.  DCN_OK or DCN_E_INVALID. */
DCN_API int dcn_output_size(const dcn_desc* d, int32_t* Ho, int32_t* Wo);

/* Bytes of device workspace needed by dcn_forward / dcn_backward (0 on invalid desc). */
DCN_API size_t dcn_forward_workspace_size(const dcn_desc* d);
DCN_API size_t dcn_backward_workspace_size(const dcn_desc* d);

/* y = DCNv2(input; weight, mask, offset, bias).  Replaces MyDCN_forward
 * (reference name.h:15-24).  workspace: >= dcn_forward_workspace_size bytes,
 * 256-byte aligned. */
DCN_API int dcn_forward(const dcn_desc* d, const void* input, const void* weight, const void* mask,
                const void* offset, const void* bias, void* output, void* workspace,
                size_t workspace_bytes, void* stream);

/* Gradients of DCNv2.  Replaces MyDCN_backward (reference name.h:26-36); the
 * outputs are the reference's return list (grad_input, grad_offset, grad_mask,
 * grad_weight, grad_bias, com.cu:845-847), each overwritten (not accumulated).
 * grad_bias may be NULL when has_bias == 0. */
DCN_API int dcn_backward(const dcn_desc* d, const void* input, const void* weight, const void* mask,
                 const void* offset, const void* bias, const void* grad_output, void* grad_input,
                 void* grad_offset, void* grad_mask, void* grad_weight, void* grad_bias,
                 void* workspace, size_t workspace_bytes, void* stream);

/* DCNv2 fed by the raw output of the offset/mask predictor conv.  Replaces the
 * reference module's chunk / cat / sigmoid between its predictor and the op
 * (dcn_v2_mm.py:133-137, DCN.forward): offset_mask is [B][3*dg*K2][Ho][Wo],
 * channels 0 .. 2*dg*K2-1 are the offsets in the op's order (the reference's
 * cat(o1, o2)) and channels 2*dg*K2 .. 3*dg*K2-1 the mask logits, which the
 * kernels pass through a sigmoid.  Same workspace and result as dcn_forward. */
DCN_API int dcn_forward_om(const dcn_desc* d, const void* input, const void* weight,
                           const void* offset_mask, const void* bias, void* output, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Gradients of dcn_forward_om: grad_offset_mask has the layout of offset_mask
 * (offset gradients, then the gradients of the mask logits, i.e. grad_mask *
 * s * (1 - s) with s the sigmoid); the other outputs as dcn_backward. */
DCN_API int dcn_backward_om(const dcn_desc* d, const void* input, const void* weight,
                            const void* offset_mask, const void* bias, const void* grad_output,
                            void* grad_input, void* grad_offset_mask, void* grad_weight, void* grad_bias,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Forward pass that allocates nothing and takes no workspace.  No counterpart
 * in the reference.  For callers that may not allocate GPU memory at all (code
 * running while a framework records a stream into a graph and forbids
 * allocation, runtimes whose memory is fixed at start-up, plugins whose host
 * owns every buffer): same arguments and result as dcn_forward minus the
 * workspace.  Scratch comes from one array of DCN_NOALLOC_SCRATCH_BYTES in the
 * library's device memory, held on every GPU that loads the library until the
 * process exits.  Problems whose dcn_forward_workspace_size exceeds that size
 * are rejected with DCN_E_SCRATCH_LIMIT.  The first call on a device looks up
 * the array's device address (make that first call before any stream capture).
 * All calls share the array, so calls that overlap on the GPU race; serialise
 * them.  Device error bits of the last call are not readable through this
 * entry point (it exposes no workspace); errors found on the host are returned. */
#define DCN_NOALLOC_SCRATCH_BYTES (48u << 20) /* 48 MiB */
DCN_API int dcn_forward_noalloc(const dcn_desc* d, const void* input, const void* weight,
                                const void* mask, const void* offset, const void* bias,
                                void* output, void* stream);

/* Synchronises `stream`, returns the device error bits recorded in `workspace`
 * by the last dcn_forward / dcn_backward that used it, and clears them.
 * Returns a negative DCN_E* code if reading them failed. */
DCN_API int dcn_read_device_status(void* workspace, void* stream);

/* Human-readable text for a DCN_* return code. */
DCN_API const char* dcn_strerror(int code);

/* Kernel timing trace (no counterpart in the reference, which only times its
 * forward inside a hard-coded benchmark loop, com_2buffer_cpasyc.cu:301-388).
 * When enabled, every kernel the library launches is bracketed by CUDA events
 * on its launch stream.  dcn_trace_collect synchronises those events and
 * returns per-kernel aggregates since the last reset: the number of entries
 * (at most max_entries are written) or a negative DCN_E* code. */
typedef struct dcn_trace_entry {
  const char* name;   /* kernel name, static storage */
  int64_t launches;   /* launches recorded */
  double total_ms;    /* summed event-to-event time */
} dcn_trace_entry;
DCN_API int dcn_trace_enable(int on);
DCN_API int dcn_trace_collect(dcn_trace_entry* out, int max_entries);
DCN_API int dcn_trace_reset(void);

/* Library version string, e.g. "dcn_b200 0.1.0 sm_100a". */
DCN_API const char* dcn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DCN_B200_H */
