/*
 * hyfft.h — C ABI of the B200-native Hyena FFT-convolution backend.
 *
 * This is the drop-in boundary for nvSubquadratic's long-convolution hot path.
 * Every entry point takes plain pointers and sizes, enqueues its work on the
 * caller's CUDA stream, allocates nothing (all scratch comes from the
 * caller-provided workspace), never throws, and returns an HYFFT_* status.
 *
 * Reference interfaces each group replaces (nvSubquadratic, file:line):
 *
 *   hyfft_conv_forward / hyfft_conv_backward
 *     the op contract  fn(x, kernel, shortcut) -> y  and its autograd backward:
 *       causal_fftconv1d_fp32_bhl   nvsubquadratic/ops/fftconv.py:546-600
 *       fftconv1d_fp32_bhl          nvsubquadratic/ops/fftconv.py:603-659
 *       fftconv2d_fp32_bhl          nvsubquadratic/ops/fftconv.py:662-733
 *       fftconv3d_fp32_bhl          nvsubquadratic/ops/fftconv.py:736-812
 *       *_fp32_blh / *_w_reshape    nvsubquadratic/ops/fftconv.py:163-538 (layout = BLH)
 *     and the external-kernel slot the reference binds for fft_backend="subq_ops"
 *       fftconv2d_bhl / causal_fftconv1d_bhl  nvsubquadratic/ops/fftconv_custom.py:133-160, :307-335
 *
 *   hyfft_hyena_forward / hyfft_hyena_backward
 *     the fused mixer  Hyena.forward(q, k, v)  with identity norms:
 *       nvsubquadratic/modules/hyena_nd.py:432-583 (short conv :505-516, gate 1 :546,
 *       global conv :563 -> modules/ckconv_nd.py:1006-1062, gate 2 :570)
 *
 *   hyfft_cp_pack / hyfft_cp_unpack
 *     the local permutations around the context-parallel all-to-all:
 *       all_to_all_single_fn  nvsubquadratic/parallel/a2a_comms.py:125-285
 *
 * Threading: the host calls are reentrant; concurrent calls on different
 * streams must use different workspaces.
 */
#ifndef HYFFT_H_
#define HYFFT_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HYFFT_API __attribute__((visibility("default")))
#else
#define HYFFT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define HYFFT_OK 0
#define HYFFT_ERR_INVALID 1      /* bad argument (shape, pointer, enum)        */
#define HYFFT_ERR_UNSUPPORTED 2  /* valid request this backend does not cover  */
#define HYFFT_ERR_WORKSPACE 3    /* workspace / saved buffer too small          */
#define HYFFT_ERR_CUDA 4         /* a CUDA launch failed (see hyfft_last_error) */

/* ---------------------------------------------------------------- enums */
#define HYFFT_F32 0
#define HYFFT_BF16 1
#define HYFFT_F16 2

#define HYFFT_LAYOUT_BHL 0 /* [B, H, *S] channels-first */
#define HYFFT_LAYOUT_BLH 1 /* [B, *S, H] channels-last  */

#define HYFFT_GATE_IDENTITY 0
#define HYFFT_GATE_SIGMOID 1
#define HYFFT_GATE_SILU 2

/* ---------------------------------------------------------------- op level */
typedef struct hyfft_conv_desc {
  int32_t ndim;         /* spatial rank: 1, 2 or 3                                  */
  int32_t batch;        /* B                                                        */
  int32_t channels;     /* H                                                        */
  int32_t n[3];         /* spatial extents (unused entries ignored)                 */
  int32_t k[3];         /* kernel extents, k[d] <= 2 * n[d]                         */
  int32_t kernel_batch; /* 1 (shared kernel) or B (per-sample / FiLM kernels)       */
  int32_t causal;       /* 1: causal 1D conv (fftconv.py:546); 0: centred "same"    */
  int32_t dtype;        /* HYFFT_F32 / BF16 / F16: dtype of x, y, shortcut, dx, dy  */
  int32_t layout;       /* HYFFT_LAYOUT_BHL or HYFFT_LAYOUT_BLH for x, y, dx, dy    */
  int32_t periodic;     /* bit d set: axis d is circular (FFT length n[d], a power   */
                        /* of two, k[d] <= n[d], output aligned by (k[d] - 1) / 2):  */
                        /* circular_fftconv{1,2,3}d_fp32_bhl ops/circular_fftconv.py */
                        /* :310-583; mixed axes ops/mixed_fftconv.py:504-723. 0: all */
                        /* axes zero-padded (the fftconv.py ops above)               */
} hyfft_conv_desc;

/* Workspace bytes for one forward / one backward call. */
HYFFT_API int hyfft_conv_workspace_size(const hyfft_conv_desc* d, size_t* fwd_bytes, size_t* bwd_bytes);

/* y = conv(x, kernel) rounded to dtype, then + shortcut * x (if shortcut != NULL).
 * x, y: contiguous in `layout`; kernel: float32 contiguous [kernel_batch, H, *k]
 * (BHL) or [kernel_batch, *k, H] (BLH); shortcut: [H] of `dtype` or NULL.          */
HYFFT_API int hyfft_conv_forward(const hyfft_conv_desc* d, const void* x, const float* kernel,
                       const void* shortcut, void* y, void* workspace, size_t workspace_bytes,
                       void* stream);

/* hyfft_conv_forward without a caller workspace and without allocating anything.
 * No counterpart in the reference (its op allocates through torch on every call).
 *
 * For callers that cannot allocate device memory at call time: an FFI binding with
 * no device allocator of its own (a ctypes / cgo / JNI caller handing over raw
 * pointers), a serving loop or pre-planned memory pool that forbids allocator
 * calls after warm-up, or code that must not grow the device footprint mid-run.
 * The scratch is one fixed array of HYFFT_CONV_SCRATCH_MAX_BYTES in the library's
 * device image, one per device; channels are processed in chunks that fit it.
 *
 * - The first call on a device looks up that array's address for the device (with
 *   the device that owns x current) and keeps it for the life of the process; make
 *   that first call before any stream capture on the device. A device reset
 *   (cudaDeviceReset, or tearing down and re-creating the primary context) can move
 *   the array, so this entry point does not support calls after a reset.
 * - It always runs the chunked pass chain, also for the 2D shapes that
 *   hyfft_conv_forward sends to its large-grid kernels; results agree within the
 *   tolerance of the dtype, not bit for bit.
 * - Problems whose single-channel spectra (plus the [H] float shortcut vector) do
 *   not fit in HYFFT_CONV_SCRATCH_MAX_BYTES are rejected with HYFFT_ERR_WORKSPACE
 *   before anything is launched; use hyfft_conv_forward with a workspace for them.
 * - Nothing in the scratch needs to start at zero: every byte a call reads was
 *   written earlier in the same call.
 * - All calls on one device share the one array: calls that overlap in time (on
 *   different streams, or from different host threads) race and corrupt each
 *   other's results. Serialize them, e.g. issue them on one stream.
 * Arguments and results are those of hyfft_conv_forward.                         */
#define HYFFT_CONV_SCRATCH_MAX_BYTES (32u << 20)
HYFFT_API int hyfft_conv_forward_static_scratch(const hyfft_conv_desc* d, const void* x, const float* kernel,
                                                const void* shortcut, void* y, void* stream);

/* Gradients of hyfft_conv_forward for upstream dy: dx (dtype, layout of x),
 * dkernel (float32, layout of kernel), dshortcut (float32 [H]; NULL when
 * shortcut is NULL). Any of dx / dkernel / dshortcut may be NULL to skip it.     */
HYFFT_API int hyfft_conv_backward(const hyfft_conv_desc* d, const void* x, const float* kernel,
                        const void* shortcut, const void* dy, void* dx, float* dkernel,
                        float* dshortcut, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- fused mixer */
typedef struct hyfft_hyena_desc {
  int32_t ndim;            /* spatial rank 1..3                                       */
  int32_t batch;           /* B                                                       */
  int32_t channels;        /* C (q, k, v each have C channels)                        */
  int32_t n[3];            /* spatial extents                                         */
  int32_t k[3];            /* long filter extents (filter is float32 [1, C, *k])      */
  int32_t causal;          /* causal long conv (1D)                                   */
  int32_t short_k[3];      /* depthwise short conv extents; 0 = no short conv         */
  int32_t short_causal;    /* 1D causal short conv (left pad short_k - 1)             */
  int32_t short_bias;      /* short conv has a bias [3C]                              */
  int32_t gate1;           /* HYFFT_GATE_* applied to k: z = q * gate1(k)             */
  int32_t gate2;           /* HYFFT_GATE_* applied to v: y = h * gate2(v)             */
  int32_t dtype;           /* activation dtype of q, k, v, y, dq, dk, dv, dy          */
  int64_t in_batch_stride; /* element strides of q, k, v and of their gradients       */
  int64_t in_pos_stride;   /*   dq, dk, dv (channel stride is 1): e.g. 3C for views    */
                           /*   into one [B, *S, 3C] projection and its gradient       */
  int64_t out_batch_stride;/* element strides of y and dy (channel stride 1)          */
  int64_t out_pos_stride;
  int32_t periodic;        /* circular axes of the long conv, as hyfft_conv_desc      */
} hyfft_hyena_desc;

/* Workspace bytes for forward / backward, and the bytes of the `saved` buffer the
 * forward fills for the backward (0 when the backward recomputes everything).   */
HYFFT_API int hyfft_hyena_workspace_size(const hyfft_hyena_desc* d, size_t* fwd_bytes, size_t* bwd_bytes,
                               size_t* saved_bytes);

/* y = gate2(v') * (conv(z) + D * z), z = q' * gate1(k'), (q', k', v') = short conv of
 * (q, k, v). filt: float32 [1, C, *k]; D: float32 [C]; short_w: float32 [3C, *short_k];
 * short_b: float32 [3C] or NULL. `saved` may be NULL when saved_bytes == 0.        */
HYFFT_API int hyfft_hyena_forward(const hyfft_hyena_desc* d, const void* q, const void* k, const void* v,
                        const float* filt, const float* D, const float* short_w,
                        const float* short_b, void* y, void* saved, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Gradients for upstream dy (read with the out strides). dq, dk, dv are written with
 * the in strides, so the gradient of a packed [B, *S, 3C] projection is one buffer.
 * dfilt [1, C, *k], dD [C], dshort_w [3C, *short_k], dshort_b [3C] are float32 and
 * OVERWRITTEN (not accumulated). `saved` is what the matching forward wrote.       */
HYFFT_API int hyfft_hyena_backward(const hyfft_hyena_desc* d, const void* q, const void* k, const void* v,
                         const float* filt, const float* D, const float* short_w,
                         const float* short_b, const void* dy, void* dq, void* dk, void* dv,
                         float* dfilt, float* dD, float* dshort_w, float* dshort_b,
                         const void* saved, void* workspace, size_t workspace_bytes,
                         void* stream);

/* ---------------------------------------------------------------- context parallel */
/* Local permutations around NCCL all_to_all_single for a 1D/2D/3D tensor whose
 * axis 2 is the sequence (a2a_comms.py:171-282). elem_bytes: 2 or 4.
 *
 * hyfft_cp_pack_split_to_full:   src [B, C, l, *rest] (rank-local, zigzag chunks)
 *                                -> dst [P, B, C/P, l, *rest] (send buffer)
 * hyfft_cp_unpack_split_to_full: src [P, B, C/P, l, *rest] (received)
 *                                -> dst [B, C/P, P*l, *rest] natural order
 *                                (inverse zigzag when zigzag != 0)
 * hyfft_cp_pack_full_to_split:   src [B, d, L, *rest] -> dst [P, B, d, L/P, *rest]
 *                                (zigzag chunk order when zigzag != 0)
 * hyfft_cp_unpack_full_to_split: src [P, B, d, l, *rest] -> dst [B, P*d, l, *rest]
 * rest = product of trailing extents after the sequence axis (1 for 1D).           */
HYFFT_API int hyfft_cp_pack_split_to_full(const void* src, void* dst, int64_t B, int64_t C, int64_t l,
                                int64_t rest, int32_t P, int32_t elem_bytes, void* stream);
HYFFT_API int hyfft_cp_unpack_split_to_full(const void* src, void* dst, int64_t B, int64_t d, int64_t l,
                                  int64_t rest, int32_t P, int32_t zigzag, int32_t elem_bytes,
                                  void* stream);
HYFFT_API int hyfft_cp_pack_full_to_split(const void* src, void* dst, int64_t B, int64_t d, int64_t L,
                                int64_t rest, int32_t P, int32_t zigzag, int32_t elem_bytes,
                                void* stream);
HYFFT_API int hyfft_cp_unpack_full_to_split(const void* src, void* dst, int64_t B, int64_t d, int64_t l,
                                  int64_t rest, int32_t P, int32_t elem_bytes, void* stream);

/* Channels-last form used by the fused CP mixer: tensors [B, seq, *rest, G, C] with the
 * sequence split along its first spatial axis (l rows per rank; zigzag chunks r and
 * 2P-1-r of 2P when zigzag != 0) and G channel groups (G = 3 moves q, k, v of one
 * [B, seq, *rest, 3C] projection output at once). d = C / P.
 *   PACK_SEQ_TO_CHAN    [B, l, rest, G, C]     -> send [P, B, l, rest, G, d]
 *   UNPACK_SEQ_TO_CHAN  recv [P, B, l, rest, G, d] -> [B, P*l, rest, G, d] (natural order)
 *   PACK_CHAN_TO_SEQ    [B, P*l, rest, G, d]  -> send [P, B, l, rest, G, d]
 *   UNPACK_CHAN_TO_SEQ  recv [P, B, l, rest, G, d] -> [B, l, rest, G, C]                */
#define HYFFT_CP_PACK_SEQ_TO_CHAN 0
#define HYFFT_CP_UNPACK_SEQ_TO_CHAN 1
#define HYFFT_CP_PACK_CHAN_TO_SEQ 2
#define HYFFT_CP_UNPACK_CHAN_TO_SEQ 3
HYFFT_API int hyfft_cp_permute_cl(const void* src, void* dst, int32_t op, int64_t B, int64_t l_rows, int64_t rest,
                                  int64_t G, int64_t C, int32_t P, int32_t zigzag, int32_t elem_bytes,
                                  void* stream);

/* The full-C side of the channels-last exchange for a window of every rank's channel
 * block, so that a caller can move the channels in groups and overlap each group's
 * all-to-all with the computation on another group (the reference moves the whole
 * tensor in one all_to_all_single, a2a_comms.py:194 and :277).
 *   PACK_SEQ_TO_CHAN    [B, l, rest, G, C] -> send [P, B, l, rest, G, c_cnt]: for every
 *                       destination rank j, channels [j*C/P + c_off, j*C/P + c_off + c_cnt)
 *   UNPACK_CHAN_TO_SEQ  recv [P, B, l, rest, G, c_cnt] -> those channels of [B, l, rest, G, C]
 *                       (the other channels of dst are left as they are)
 * 0 <= c_off, c_off + c_cnt <= C/P. The channel-block side of the same exchange is
 * hyfft_cp_permute_cl with C = c_cnt * P.                                           */
HYFFT_API int hyfft_cp_permute_cl_window(const void* src, void* dst, int32_t op, int64_t B, int64_t l_rows,
                                         int64_t rest, int64_t G, int64_t C, int32_t P, int64_t c_off,
                                         int64_t c_cnt, int32_t elem_bytes, void* stream);

/* ---------------------------------------------------------------- direct causal conv */
/* Depthwise causal 1D convolution computed directly (no FFT), for short and medium
 * filters (K <= 1024), channel-major [B, C, L] activations of `dtype`:
 *   y = act(round(conv)),  conv[b, c, t] = sum_{k < K} w[c, k] x[b, c, t - (K - 1) + k] + bias[c]
 * (x = 0 before t = 0), act = identity (activation 0) or SiLU (activation 1).
 * Replaces the external kernel the reference binds in
 *   causal_conv1d        nvsubquadratic/ops/causal_conv1d_custom.py:81-98
 *   SubqOpsCausalConv1d  nvsubquadratic/modules/subq_ops_causal_conv1d.py:36-83
 * weight: float32 [C, K]; bias: float32 [C] or NULL.                                  */
HYFFT_API int hyfft_causal_conv1d_forward(const void* x, const float* weight, const float* bias, void* y,
                                          int64_t B, int64_t C, int64_t L, int32_t K, int32_t activation,
                                          int32_t dtype, void* stream);
/* Gradients for upstream dy: dx ([B, C, L] of dtype), dweight (float32 [C, K]) and dbias
 * (float32 [C], NULL to skip); dweight and dbias are overwritten.                      */
HYFFT_API int hyfft_causal_conv1d_backward(const void* x, const float* weight, const float* bias, const void* dy,
                                           void* dx, float* dweight, float* dbias, int64_t B, int64_t C, int64_t L,
                                           int32_t K, int32_t activation, int32_t dtype, void* stream);

/* ---------------------------------------------------------------- implicit filter (SIREN)
 * The filter generator of the Hyena long convolution: a SIREN network evaluated on the
 * coordinate grid, then the exponential window, in float32 (replaces
 * nvsubquadratic/modules/kernels_nd.py SIRENKernelND.forward :1149-1199 with its positional
 * embedding :818-874, no FiLM, and masks_nd.py ExponentialModulationND.forward :229-255).
 *
 *   h0 = sin(pe_w x + pe_b); h_l = sin(W_l h_{l-1} + b_l), l = 1..num_hidden;
 *   k[p, c] = (out_w h + out_b)[c] * prod_d exp(-|x_d(p)| |mask_w[d, c]|)
 *
 * coords: the per-axis coordinate vectors concatenated (n[0] + .. + n[ndim-1] floats, the
 * reference's sliced linspace grid); points are row-major over the axes (G = prod n).
 * Weights: pe_w [E, ndim], pe_b [E] | NULL, hid_w the hidden layers' weights concatenated
 * ([H, E] then num_hidden - 1 times [H, H]), hid_b [num_hidden, H] | NULL, out_w [C, H],
 * out_b [C] | NULL, mask_w [ndim, C] | NULL (no window). kernel: [G, C] (layout BLH, the
 * reference's [1, *S, C]) or [C, G] (layout BHL, the mixer's [1, C, *S]). saved: G * H
 * floats written by the forward and read by the backward; workspace: G * H floats.
 * The backward overwrites every gradient it is given; mask_w gets none (fixed window).
 * E, H <= 128 (HYFFT_ERR_UNSUPPORTED above, or when the backward's shared memory would
 * exceed a CTA's). */
typedef struct hyfft_siren_desc {
  int32_t ndim;        /* 1..3 */
  int32_t n[3];        /* grid points per axis (2 * seq_len - 1 in the reference) */
  int32_t embedding;   /* E */
  int32_t hidden;      /* H */
  int32_t num_hidden;  /* hidden linear layers (the reference's num_layers - 1), >= 1 */
  int32_t channels;    /* C */
  int32_t layout;      /* HYFFT_LAYOUT_BLH: kernel [G, C]; HYFFT_LAYOUT_BHL: [C, G] */
} hyfft_siren_desc;

HYFFT_API int hyfft_siren_sizes(const hyfft_siren_desc* d, size_t* saved_bytes, size_t* workspace_bytes);
HYFFT_API int hyfft_siren_forward(const hyfft_siren_desc* d, const float* coords, const float* pe_w,
                                  const float* pe_b, const float* hid_w, const float* hid_b, const float* out_w,
                                  const float* out_b, const float* mask_w, float* kernel, void* saved,
                                  size_t saved_bytes, void* stream);
HYFFT_API int hyfft_siren_backward(const hyfft_siren_desc* d, const float* coords, const float* pe_w,
                                   const float* pe_b, const float* hid_w, const float* hid_b, const float* out_w,
                                   const float* mask_w, const float* dkernel, const void* saved, float* d_pe_w,
                                   float* d_pe_b, float* d_hid_w, float* d_hid_b, float* d_out_w, float* d_out_b,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- misc */
/* Message of the most recent error on this thread ("" if none). */
HYFFT_API const char* hyfft_last_error(void);
/* Library version string. */
HYFFT_API const char* hyfft_version(void);
/* Number of kernels this process has launched through the library so far. */
HYFFT_API long long hyfft_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* HYFFT_H_ */
