/*
 * C ABI of the B200-native ICTC-O2 tensor-product kernels (libictc_o2_b200.so).
 *
 * Every entry point takes plain device pointers and sizes, launches on the
 * given CUDA stream (NULL = legacy default stream), never aborts, and returns
 * an ICTC status code; ictc_o2_last_error() gives a message for the calling
 * thread.  All tensors are contiguous row-major FP32.  The library allocates
 * no device memory in these entry points: callers pass outputs and workspace.
 *
 * The functions replace the reference's Triton custom ops (paths relative to
 * the reference project root); path metadata tensors and the process-global
 * metadata registry of the reference become (channels, m_max, parity,
 * normalization) integers, from which the library derives its compiled tables.
 */
#ifndef ICTC_O2_B200_H_
#define ICTC_O2_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ICTC_API __attribute__((visibility("default")))
#else
#define ICTC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ICTC_OK = 0,
  ICTC_ERR_INVALID = 1,      /* bad argument: size, null pointer, alignment */
  ICTC_ERR_UNSUPPORTED = 2,  /* configuration without a compiled kernel */
  ICTC_ERR_CUDA = 3,         /* CUDA launch or runtime error */
  ICTC_ERR_WORKSPACE = 4     /* workspace smaller than the queried size */
};

enum { ICTC_PARITY_CANONICAL = 0, ICTC_PARITY_FULL = 1 };
enum { ICTC_NORM_COMPONENT = 0, ICTC_NORM_NORM = 1 };
/* Storage order inside the frequency blocks of a TensorProduct row:
 * [copy][channel][component] (TensorProduct, layout 0 of triton_o2.py:111-113) or
 * [copy][component][channel] (ComponentMajorTensorProduct, layouts 1 / 2 of
 * triton_o2.py:114-118, triton_o2.py:1204-1278). */
enum { ICTC_LAYOUT_CHANNEL_MAJOR = 0, ICTC_LAYOUT_COMPONENT_MAJOR = 1 };

/* Message describing the last non-OK status returned on this thread. */
ICTC_API const char* ictc_o2_last_error(void);

/* Library ABI version (major * 100 + minor). */
ICTC_API int32_t ictc_o2_abi_version(void);

/* Synchronizes with the current device, then reads and clears the kernels'
 * device-side error flags (one per compiled unit: TensorProduct, uvu, radial and
 * the wait probe below) and returns the first nonzero code in that order: 0 = none;
 * nonzero = a bounded wait inside a kernel ran out (2 s of the GPU's global timer)
 * and that kernel stopped early, so its outputs are invalid.  Codes: 1-4
 * TensorProduct staged kernels (stage ring, drain, weight copy), 5-6 radial edge
 * tile, 7-8 shared-weight uvu tile, 9-10 per-row uvu streamed kernel, 11-12
 * per-row uvu quad kernel, 13 the wait probe; 17 is not a wait: a gathered radial
 * call met a node index out of range.  No counterpart in the reference,
 * whose Triton kernels have no waits. */
ICTC_API int32_t ictc_o2_device_error(int32_t* code);

/* Test hook, no counterpart in the reference: launches one CTA that waits, with the
 * kernels' bounded-wait helper and a limit of `limit_us` microseconds (1 to
 * 1,000,000), on an mbarrier that nothing arrives at.  The wait runs out, the CTA
 * records code 13 in the device error flag and exits; *waited_ok (a device int)
 * receives 0.  Read the code with ictc_o2_device_error. */
ICTC_API int32_t ictc_o2_test_wait_timeout(int32_t limit_us, int32_t* waited_ok,
                                           void* stream);

/* ---------------------------------------------------------------- TensorProduct
 * Flat channel-major operands of width W = C * (2 * m_max + 1) * (full ? 2 : 1),
 * layout [0e: C][0o: C (full)][m = 1..m_max: copy (1 or 2) x C x 2]
 * (reference: src/ictc_o2_hp/api.py:43-54, triton_o2.py:1169-1201).
 */

/* Packed weight length (reference: fast_o2.py:152-167, native_o2.py:101-117). */
ICTC_API int32_t ictc_o2_tp_weight_numel(int32_t channels, int32_t m_max, int32_t parity,
                                int64_t* numel);

/* Compiled path table, for host-side consistency checks: for each block path,
 * 7 + 4 * 4 int32 = {in1 slot, in2 slot, out slot, class, unit offset, copied,
 * nterms, then 4 x (i, j, k, sign)}.  `count` receives the path count. */
ICTC_API int32_t ictc_o2_tp_path_table(int32_t m_max, int32_t parity, int32_t* table,
                              int32_t capacity_paths, int32_t* count);

/* out[N, W] = TP(left, right; weight).  Replaces the o2_forward custom op
 * (reference: src/ictc_o2_hp/triton_o2.py:786-875). */
ICTC_API int32_t ictc_o2_tp_forward(const float* left, const float* right, const float* weight,
                           float* output, int64_t rows, int32_t channels, int32_t m_max,
                           int32_t parity, int32_t normalization, void* stream);

/* ictc_o2_tp_forward with the frequency-block storage order `layout`
 * (ICTC_LAYOUT_*): component-major rows are read and written in place, the
 * metadata layout field of the reference's o2_forward (triton_o2.py:786-794). */
ICTC_API int32_t ictc_o2_tp_forward_layout(const float* left, const float* right,
                                  const float* weight, float* output, int64_t rows,
                                  int32_t channels, int32_t m_max, int32_t parity,
                                  int32_t normalization, int32_t layout, void* stream);

/* Workspace bytes needed by ictc_o2_tp_backward on `device` for these sizes. */
ICTC_API int32_t ictc_o2_tp_backward_workspace(int64_t rows, int32_t channels, int32_t m_max,
                                      int32_t parity, int32_t device, size_t* bytes);

/* Full first-order VJP: grad_left, grad_right [N, W] and grad_weight [numel]
 * (deterministic fixed-order reduction over rows).  Replaces the o2_backward
 * custom op (reference: src/ictc_o2_hp/triton_o2.py:878-966); N = 0 writes a
 * zero grad_weight (triton_o2.py:890-891). */
ICTC_API int32_t ictc_o2_tp_backward(const float* left, const float* right, const float* weight,
                            const float* grad_output, float* grad_left, float* grad_right,
                            float* grad_weight, void* workspace, size_t workspace_bytes,
                            int64_t rows, int32_t channels, int32_t m_max, int32_t parity,
                            int32_t normalization, void* stream);

/* ictc_o2_tp_backward with the frequency-block storage order `layout` (reference
 * o2_backward, triton_o2.py:878-887, on layout-1/2 metadata); the workspace is the
 * same as for ictc_o2_tp_backward. */
ICTC_API int32_t ictc_o2_tp_backward_layout(const float* left, const float* right,
                                   const float* weight, const float* grad_output,
                                   float* grad_left, float* grad_right, float* grad_weight,
                                   void* workspace, size_t workspace_bytes, int64_t rows,
                                   int32_t channels, int32_t m_max, int32_t parity,
                                   int32_t normalization, int32_t layout, void* stream);

/* ictc_o2_tp_backward for callers that cannot allocate device memory (their
 * allocator belongs to a host runtime or a memory pool they must not bypass, or
 * device memory was reserved up front): no counterpart in the reference.  Same
 * kernels and results as ictc_o2_tp_backward; the workspace is a fixed 32 MiB
 * array in device memory owned by the library, held on every GPU that loads it.
 * Sizes whose workspace (ictc_o2_tp_backward_workspace) exceeds 32 MiB return
 * ICTC_ERR_WORKSPACE.  The first call on a device looks up the array's device
 * address; make it before any stream capture.  Calls share the array: calls
 * that overlap on the GPU race and must be ordered by the caller.  Nothing in
 * the array needs clearing between calls.  Allocates no memory. */
ICTC_API int32_t ictc_o2_tp_backward_noalloc(const float* left, const float* right,
                                    const float* weight, const float* grad_output,
                                    float* grad_left, float* grad_right, float* grad_weight,
                                    int64_t rows, int32_t channels, int32_t m_max,
                                    int32_t parity, int32_t normalization, void* stream);

/* ------------------------------------------------------------ UvuTensorProduct
 * First input / output: C channels per representation copy, flat
 * [copy, channel, component] blocks; second input: V channels per copy
 * (reference: src/ictc_o2_hp/uvu_o2.py:27-41, 76-156).  Configuration arguments,
 * shared by the entry points below:
 *   channels (C), channels_in2 (V), m_max, parity, m_max_in2, parity_in2,
 *   normalization, path_normalization (0 = none, 1 = element/path; they coincide
 *   for this API, uvu_o2.py:138-144).
 * The path table is built by the library (ictc_o2_uvu_table); the caller copies
 * it once to the device and passes that pointer, the role of the reference's
 * path_info / coefficients buffers (uvu_triton.py:39-67). */

/* Packed path table (int32 words, coefficients stored as float bits): a 16-word
 * header {n_in1, n_in2, n_paths, C, V, width1, width2, 0, then the word offsets
 * of the sections below and the total words}, then (offset, dim) per entry of
 * each input, (i, j, k, 0) per path, 8 coefficients c[k][a][b] per path, and the
 * paths ordered by first and by second entry; each section starts on a 16-byte
 * boundary.  With table == NULL only `words` is written. */
ICTC_API int32_t ictc_o2_uvu_table(int32_t channels, int32_t channels_in2, int32_t m_max,
                                   int32_t parity, int32_t m_max_in2, int32_t parity_in2,
                                   int32_t normalization, int32_t path_normalization,
                                   int32_t* table, int64_t capacity_words, int64_t* words);

/* Workspace bytes of the forward and backward entry points (device `device`). */
ICTC_API int32_t ictc_o2_uvu_workspace(int32_t channels, int32_t channels_in2, int32_t m_max,
                                       int32_t parity, int32_t m_max_in2, int32_t parity_in2,
                                       int32_t normalization, int32_t path_normalization,
                                       int32_t shared, int64_t rows, int32_t device,
                                       size_t* forward_bytes, size_t* backward_bytes);

/* out[N, width1].  weight: [weight_numel] when shared, else [N, weight_numel].
 * Replaces the uvu forward / forward_into ops (reference: uvu_triton.py:235-284). */
ICTC_API int32_t ictc_o2_uvu_forward(const float* left, const float* right, const float* weight,
                                     float* output, int64_t rows, int32_t channels,
                                     int32_t channels_in2, int32_t m_max, int32_t parity,
                                     int32_t m_max_in2, int32_t parity_in2,
                                     int32_t normalization, int32_t path_normalization,
                                     int32_t shared, const void* device_table, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* VJP; `needed` is the role mask 1 = grad_left, 2 = grad_right, 4 = grad_weight
 * (the reference's `needed`, uvu_triton.py:18-36, 287-414).  grad_weight is
 * [weight_numel] (shared, summed over rows in a fixed order) or [N, weight_numel]. */
ICTC_API int32_t ictc_o2_uvu_backward(const float* left, const float* right, const float* weight,
                                      const float* grad_output, float* grad_left,
                                      float* grad_right, float* grad_weight, int64_t rows,
                                      int32_t channels, int32_t channels_in2, int32_t m_max,
                                      int32_t parity, int32_t m_max_in2, int32_t parity_in2,
                                      int32_t normalization, int32_t path_normalization,
                                      int32_t shared, int32_t needed, const void* device_table,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------ RadialUvuTensorProduct
 * out = uvu(left, angular, hidden @ alpha^T + bias) with a V = 1 per-edge uvu
 * (reference: src/ictc_o2_hp/radial_uvu.py:21-66, radial_streamed.py:37-146).
 * Shapes: left [N, width1], angular [N, width2], hidden [N, H], alpha [P*C, H],
 * bias [P*C] or NULL.  The edge weights are regenerated on chip and never
 * written.  Configuration: channels (C <= 128), m_max, parity, m_max_in2,
 * parity_in2, normalization, path_normalization, hidden (H); the device table
 * is ictc_o2_uvu_table(channels, 1, ...) copied to the device. */

ICTC_API int32_t ictc_o2_radial_workspace(int32_t channels, int32_t m_max, int32_t parity,
                                          int32_t m_max_in2, int32_t parity_in2,
                                          int32_t normalization, int32_t path_normalization,
                                          int32_t hidden, int64_t rows, int32_t device,
                                          size_t* forward_bytes, size_t* backward_bytes);

/* Replaces radial_stream_forward (reference: radial_streamed.py:81-99). */
ICTC_API int32_t ictc_o2_radial_forward(const float* left, const float* angular,
                                        const float* radial_hidden, const float* alpha,
                                        const float* bias, float* output, int64_t rows,
                                        int32_t channels, int32_t m_max, int32_t parity,
                                        int32_t m_max_in2, int32_t parity_in2,
                                        int32_t normalization, int32_t path_normalization,
                                        int32_t hidden, const void* device_table,
                                        void* workspace, size_t workspace_bytes, void* stream);

/* Replaces radial_stream_backward (reference: radial_streamed.py:109-139).  Role
 * mask: 1 left, 2 angular, 4 hidden, 8 alpha, 16 bias; left and angular
 * gradients are produced together (both buffers required if either is), and
 * grad_alpha is required whenever the bias gradient is.  dalpha and dbias are
 * summed over edges in a fixed order. */
ICTC_API int32_t ictc_o2_radial_backward(const float* left, const float* angular,
                                         const float* radial_hidden, const float* alpha,
                                         const float* bias, const float* grad_output,
                                         float* grad_left, float* grad_angular,
                                         float* grad_hidden, float* grad_alpha,
                                         float* grad_bias, int64_t rows, int32_t channels,
                                         int32_t m_max, int32_t parity, int32_t m_max_in2,
                                         int32_t parity_in2, int32_t normalization,
                                         int32_t path_normalization, int32_t hidden,
                                         int32_t needed, const void* device_table,
                                         void* workspace, size_t workspace_bytes, void* stream);

/* The radial product with the node gather folded into its first input (no
 * counterpart in the reference, whose chain starts at per-edge inputs,
 * docs/RADIAL.md:97-99): row e of `left` is row left_index[e] of nodes
 * [node_rows, width1], read in place by the edge kernels instead of a gathered
 * [N, width1] copy.  The backward writes the gradient of each edge's gathered row,
 * grad_left_edges [N, width1] (sum it into the nodes with ictc_o2_segment_sum over
 * the edges grouped by left_index).  Only the edge-tile kernels read gathered
 * rows: a hidden width they cannot hold, or a backward request without the left /
 * angular roles but with hidden, alpha or bias, answers ICTC_ERR_UNSUPPORTED
 * (gather with ictc_o2_gather_rows and use the entries above instead).  An index
 * outside [0, node_rows) reads a zero row and sets device error code 17. */
ICTC_API int32_t ictc_o2_radial_forward_gathered(
    const float* nodes, const int64_t* left_index, int64_t node_rows, const float* angular,
    const float* radial_hidden, const float* alpha, const float* bias, float* output,
    int64_t rows, int32_t channels, int32_t m_max, int32_t parity, int32_t m_max_in2,
    int32_t parity_in2, int32_t normalization, int32_t path_normalization, int32_t hidden,
    const void* device_table, void* workspace, size_t workspace_bytes, void* stream);

ICTC_API int32_t ictc_o2_radial_backward_gathered(
    const float* nodes, const int64_t* left_index, int64_t node_rows, const float* angular,
    const float* radial_hidden, const float* alpha, const float* bias, const float* grad_output,
    float* grad_left_edges, float* grad_angular, float* grad_hidden, float* grad_alpha,
    float* grad_bias, int64_t rows, int32_t channels, int32_t m_max, int32_t parity,
    int32_t m_max_in2, int32_t parity_in2, int32_t normalization, int32_t path_normalization,
    int32_t hidden, int32_t needed, const void* device_table, void* workspace,
    size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------
 * Message-passing plumbing around the radial product (the node gather and the
 * message sum the reference leaves outside its chain, docs/RADIAL.md:97-99), with a
 * fixed summation order so that node outputs and gradients are bit-identical
 * from run to run.
 * ------------------------------------------------------------------------------ */

/* out[r, :] = source[index[r], :] for r < rows (rows of `width` floats; index into
 * [0, source_rows)).  An out-of-range index writes a zero row and raises the flag
 * read by ictc_o2_graph_bad_index. */
ICTC_API int32_t ictc_o2_gather_rows(const float* source, const int64_t* index, float* out,
                            int64_t rows, int64_t width, int64_t source_rows, void* stream);

/* out[s, :] = sum of values[order ? order[e] : e, :] for e in [offsets[s],
 * offsets[s + 1]), added in increasing e (segments = rows of out; offsets has
 * segments + 1 entries; order, when given, has value_rows entries, each in
 * [0, value_rows)).  A segment whose offsets fall outside [0, value_rows] or
 * decrease, and any out-of-range order entry, raise the flag read by
 * ictc_o2_graph_bad_index; such a segment is written as zeros.  With order = the edges
 * sorted by destination and offsets = the destinations' CSR pointers this is the
 * message sum; grouped by source, the node gradient of a gather. */
ICTC_API int32_t ictc_o2_segment_sum(const float* values, const int64_t* offsets,
                            const int64_t* order, float* out, int64_t segments, int64_t width,
                            int64_t value_rows, void* stream);

/* Synchronizes, then reads and clears the out-of-range-index flag of the two
 * kernels above on the current device (1 = some index was out of range). */
ICTC_API int32_t ictc_o2_graph_bad_index(int32_t* flag);

#ifdef __cplusplus
}
#endif

#endif /* ICTC_O2_B200_H_ */
