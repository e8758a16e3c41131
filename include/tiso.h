/*
 * tiso.h - the C ABI of torchisotonic_b200's CUDA kernels (libtiso.so, built for sm_100a).
 *
 * Plain pointers and sizes; no torch types. The caller owns every buffer: inputs, outputs and
 * a workspace sized by the *_workspace_size query. Every call is asynchronous on the given
 * CUDA stream (a cudaStream_t passed as void*; NULL is the legacy default stream), allocates
 * nothing, and returns TISO_OK or an error code whose message tiso_last_error() gives (per
 * calling thread).
 *
 * Layout: y, w, out, starts, g, grad_y, grad_w are row-major [batch, n] and contiguous; the
 * fit runs along each row. Element types: y, out, g and grad_y have the data type `dtype`
 * (TISO_F16, TISO_BF16, TISO_F32 or TISO_F64); w and grad_w the accumulation type: TISO_F64 for
 * float64 data, TISO_F32 otherwise (float16 and bfloat16 data are computed in float32, as the
 * reference does). starts is one byte per element, 1 where a block of the fit starts.
 */
#ifndef TISO_H_
#define TISO_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum tiso_status {
  TISO_OK = 0,
  TISO_ERR_ARGUMENT = 1,  /* bad shape, dtype or flag combination */
  TISO_ERR_WORKSPACE = 2, /* workspace missing or smaller than the query said */
  TISO_ERR_CUDA = 3       /* a CUDA launch or runtime call failed */
};

enum tiso_dtype { TISO_F16 = 0, TISO_BF16 = 1, TISO_F32 = 2, TISO_F64 = 3 };

enum tiso_flag {
  TISO_INCREASING = 1u, /* else a non-increasing fit */
  TISO_EXACT = 2u,      /* float32 sums kept exact (double); off: float32 sums, ~1e-3 band */
  TISO_CLIP_LO = 4u,    /* clip the fit below at y_min */
  TISO_CLIP_HI = 8u,    /* clip the fit above at y_max */
  TISO_WANT_GRAD_W = 16u /* tiso_grad: also the gradient in the weights */
};

/* Bytes of workspace tiso_fit needs for these arguments (0 when rows fit one CTA).
 * Replaces the scratch allocations of the reference's run_chunks
 * (src/torchisotonic/csrc/tiles.cuh:1762-1780), made by the caller here. */
int tiso_fit_workspace_size(int dtype, int weighted, int64_t batch, int64_t n, unsigned flags,
                            size_t* bytes);

/* The isotonic fit of every row of y, with optional weights w (NULL: unweighted), written to
 * out (clipped per flags, in dtype) and, if starts is not NULL, where its blocks start.
 * A row containing NaN is NaN throughout, with one block starting at its first element.
 * bad_weight: NULL, or a device int32 set to 1 if any weight is not > 0 (it is zeroed first).
 * Replaces torchisotonic::isotonic_tiles (schema src/torchisotonic/csrc/ops.cpp:47-49, CUDA
 * implementation src/torchisotonic/csrc/tiles.cuh:1923-1959) together with the clamp and the
 * casts around it (src/torchisotonic/_api.py:65-70) and the weight check (_api.py:60). */
int tiso_fit(int dtype, const void* y, const void* w, void* out, uint8_t* starts, int64_t batch,
             int64_t n, unsigned flags, double y_min, double y_max, int32_t* bad_weight,
             void* workspace, size_t workspace_bytes, void* stream);

/* Sets *flag (device int32; zeroed first) to 1 if any of the numel weights w (dtype TISO_F32
 * or TISO_F64) is not > 0 (NaN included): the reference's check bool((w > 0).all())
 * (src/torchisotonic/_api.py:60) as one pass of its own, so that a caller can copy the flag to
 * the host and wait for this pass alone while the fit that follows it runs. (tiso_fit's
 * bad_weight gives the same answer, but only once the whole fit is done.) */
int tiso_check_weights(int dtype, const void* w, int64_t numel, int32_t* flag, void* stream);

/* Bytes of workspace tiso_grad needs (0 when rows fit one CTA: up to 1024 elements). */
int tiso_grad_workspace_size(int dtype, int weighted, int64_t batch, int64_t n, unsigned flags,
                             size_t* bytes);

/* Gradients of sum(out * g) for out = tiso_fit(y, w, ...), from the fit's block starts:
 *   grad_y = w G / W  and, with TISO_WANT_GRAD_W, grad_w = (y - fit) G / W,
 * G and W the sums over an element's block of g (zero where clipping is active: outside
 * [y_min, y_max], bounds inclusive) and of w (1 when w is NULL). The fit (block mean of y) is
 * recomputed from y and w when the clip or grad_w needs it. y may be NULL when neither does.
 * grad_y may be NULL (not wanted). flags: TISO_CLIP_LO/HI with the bounds of the forward,
 * TISO_WANT_GRAD_W. Replaces torchisotonic::isotonic_grad (schema ops.cpp:50, CUDA
 * implementation src/torchisotonic/csrc/grad.cuh:386-413) and the clamp's and casts' backward
 * that autograd runs before it. */
int tiso_grad(int dtype, const void* y, const void* w, const uint8_t* starts, const void* g,
              void* grad_y, void* grad_w, int64_t batch, int64_t n, unsigned flags, double y_min,
              double y_max, void* workspace, size_t workspace_bytes, void* stream);

/* tiso_grad for callers that cannot allocate device memory at all - a host with no device
 * allocator of its own to hand (a plain C or foreign-language caller that links only this
 * library and the CUDA runtime), or one whose device memory is budgeted up front - and so can
 * pass no workspace. Same arguments and results as tiso_grad, without the workspace: rows of
 * more than 1024 elements use a fixed scratch array inside this library instead (4,128,768
 * bytes, 3.94 MiB: a file-scope __device__ array held by every GPU that loads the library until
 * the process exits). Limit: for such rows batch * ceil(n / 1024) <= 32768; larger problems are
 * refused with TISO_ERR_WORKSPACE (use tiso_grad). Shorter rows need no scratch and no limit.
 * The call allocates nothing. Its first call on a device looks up the array's device address
 * on that device (cudaGetSymbolAddress); make that first call before any stream capture. The
 * address is looked up again when the calling thread's current context differs from the one of
 * the last lookup on that device. A device reset (cudaDeviceReset) frees the array with its
 * context: call this function again after one only once the runtime has created the device's
 * new context, and before any capture. All calls share the one array: calls whose kernels
 * overlap on the GPU (other streams, other host threads) race on it. Nothing needs clearing
 * between calls: every scratch slot a call reads is written earlier in the same call.
 * No counterpart in the reference: an addition of this library. */
int tiso_grad_noalloc(int dtype, const void* y, const void* w, const uint8_t* starts,
                      const void* g, void* grad_y, void* grad_w, int64_t batch, int64_t n,
                      unsigned flags, double y_min, double y_max, void* stream);

/* ---- Ragged rows -----------------------------------------------------------------------------
 * Rows of different lengths packed back to back, instead of padded into [batch, n]: row r is
 * elements [offsets[r], offsets[r + 1]) of y, w, out, starts, g, grad_y and grad_w (offsets:
 * device int64[batch + 1], non-decreasing; empty rows allowed). max_len bounds every row's
 * length (at most 512): a longer row is cut to its first max_len elements - nothing beyond them
 * is read or written - so max_len must be exact or larger. No workspace is needed.
 * The reference documents ragged batches as padded rows (README.md:100-103: pad each row at its
 * end with values above its maximum); these replace that padding and the fit of the padding. */

/* tiso_fit over ragged rows (arguments and results as tiso_fit's, per row). */
int tiso_fit_varlen(int dtype, const void* y, const void* w, void* out, uint8_t* starts,
                    const int64_t* offsets, int64_t batch, int64_t max_len, unsigned flags,
                    double y_min, double y_max, int32_t* bad_weight, void* stream);

/* tiso_grad over ragged rows (arguments and results as tiso_grad's, per row). */
int tiso_grad_varlen(int dtype, const void* y, const void* w, const uint8_t* starts,
                     const void* g, void* grad_y, void* grad_w, const int64_t* offsets,
                     int64_t batch, int64_t max_len, unsigned flags, double y_min, double y_max,
                     void* stream);

/* ---- One long row split into contiguous segments across devices ----------------------------
 * The reference has no multi-device path; these replace its single-device long-row pipeline
 * (src/torchisotonic/csrc/tiles.cuh:1750-1813, run_chunks) when a row is sharded. Each device
 * holds a segment [seg_start, seg_start + seg_n) of the row and calls tiso_segment_blocks; the
 * block lists of all segments are gathered (in segment order, list k at offset k * cap, counts
 * and NaN flags per segment); each device then calls tiso_segment_expand for its own segment.
 * y0: the row's offset (every segment must pass the same value; the single-device kernels use
 * the row's first element v: v cut to 8 significant bits if |v| >= 1, else 0). Sums are double
 * (exact=True only). */

/* Workspace for tiso_segment_blocks. */
int tiso_segment_blocks_workspace_size(int dtype, int weighted, int64_t seg_n, unsigned flags,
                                       size_t* bytes);

/* The number of 512-element tiles of a segment of seg_n elements (tile_offs below has one
 * entry more). */
int tiso_segment_tile_count(int64_t seg_n, int64_t* tiles);

/* The segment's fitted blocks, in order: global first element, T (sum of sign * w * (y - y0))
 * and W (sum of w) per block, in arrays of capacity seg_n; *count (device int32) the number of
 * blocks, *nan_flag (device int32) set when the segment holds a NaN. tile_offs: NULL, or a
 * device int64 array of tiso_segment_tile_count + 1 entries, set to where each 512-element
 * tile's blocks begin in the list (every block starts in the tile it is listed under). */
int tiso_segment_blocks(int dtype, const void* y, const void* w, int64_t seg_n, int64_t seg_start,
                        unsigned flags, double y0, int64_t* blk_start, double* blk_t,
                        double* blk_w, int32_t* count, int32_t* nan_flag, int32_t* bad_weight,
                        int64_t* tile_offs, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Workspace for tiso_segment_expand (parts: number of segments, at most 32). */
int tiso_segment_expand_workspace_size(int parts, size_t* bytes);

/* Merges the gathered lists (modified in place) and writes the fit of segment `me` (clipped
 * per flags, in dtype) and, if starts is not NULL, its block starts. tile_offs: the segment's
 * tile offsets from its tiso_segment_blocks call (a CTA per tile then finds the tile's blocks
 * directly), or NULL (every element's block is searched in the whole list). */
int tiso_segment_expand(int dtype, int parts, int me, int64_t cap, int64_t* blk_start,
                        double* blk_t, double* blk_w, const int32_t* counts, const int32_t* nans,
                        int64_t seg_n, int64_t seg_start, unsigned flags, double y0, double y_min,
                        double y_max, void* out, uint8_t* starts, const int64_t* tile_offs,
                        void* workspace, size_t workspace_bytes, void* stream);

/* The backward of a split row, in two steps around an all-gather. starts, g, y, w: the
 * segment's; y0: the row's offset as in the forward. The same workspace serves both steps. */
int tiso_segment_grad_workspace_size(int dtype, int weighted, int64_t seg_n, unsigned flags,
                                     size_t* bytes);

/* Step 1: the segment's run (10 doubles, device: whether a block starts in it, then the sums
 * of g, w and w (y - y0) before its first start, from its last start on, and of all of it). */
int tiso_segment_grad_sums(int dtype, const void* y, const void* w, const uint8_t* starts,
                           const void* g, int64_t seg_n, int64_t seg_start, unsigned flags,
                           double y0, double* run, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Step 2, after the runs of all segments are gathered in order ([parts][10], device): the
 * gradients of segment `me` (the blocks reaching into it from the other segments included). */
int tiso_segment_grad(int dtype, int parts, int me, const double* runs, const void* y,
                      const void* w, const uint8_t* starts, const void* g, void* grad_y,
                      void* grad_w, int64_t seg_n, int64_t seg_start, unsigned flags, double y0,
                      double y_min, double y_max, void* workspace, size_t workspace_bytes,
                      void* stream);

/* Calibration around the fit. The reference gives these steps as torch code beside the fit:
 * fit_calibration and calibrate (README.md:43-56; examples/ctr_calibration/calibrate.py:163-186,
 * whose isotonic call is at :184). key_dtype and label_dtype: TISO_F32 or TISO_F64. */

/* Workspace for tiso_calib_groups (the sorted pairs, the radix sort's scratch, per-tile sums;
 * only the last with presorted != 0). */
int tiso_calib_groups_workspace_size(int key_dtype, int label_dtype, int64_t n, int presorted,
                                     size_t* bytes);

/* The pre-step of fit_calibration (torch.sort, unique_consecutive, index_add_, sums / counts):
 * sorts the n >= 1 (score, label) pairs by score (presorted != 0: they come sorted by score,
 * ascending, and are read in place) and pools equal scores. For the G distinct
 * scores in increasing order writes xs[g] (key_dtype), y[g] = the mean of their labels and
 * w[g] = their count (double); all three have capacity n. groups: device int64[2], set to G and
 * to 1 if a score is NaN (the outputs are then undefined). The curve is then
 * tiso_fit(TISO_F64, y, w, fit, ..., batch 1, n G, TISO_INCREASING | TISO_EXACT, ...). */
int tiso_calib_groups(int key_dtype, const void* scores, int label_dtype, const void* labels,
                      int64_t n, int presorted, void* xs, double* y, double* w, int64_t* groups,
                      void* workspace, size_t workspace_bytes, void* stream);

/* calibrate: the m scores x (key_dtype) read on the curve (xs, fit) of g >= 1 points, linear
 * between them and constant beyond, with torch's steps and roundings: i = the first index with
 * x <= xs[i] (g for NaN), clamped to [1, g - 1] (to 0 when g = 1; index -1 then means g - 1);
 * t = (x - xs[i-1]) / (xs[i] - xs[i-1]) in key_dtype, clamped to [0, 1];
 * out = fit[i-1] + t (fit[i] - fit[i-1]) in double. Needs no workspace. */
int tiso_calib_interp(int key_dtype, const void* x, int64_t m, const void* xs, const double* fit,
                      int64_t g, double* out, void* stream);

/* The message of the calling thread's last error ("" if none). */
const char* tiso_last_error(void);

/* TISO_ABI_VERSION of the library. */
int tiso_abi_version(void);

#define TISO_ABI_VERSION 2

#ifdef __cplusplus
}
#endif

#endif /* TISO_H_ */
