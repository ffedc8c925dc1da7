/*
 * B200 extensions of the C ABI. They have upstream-style conventions (0 / -1
 * and XGBGetLastError) and plain pointers and sizes.
 */
#ifndef XGB_B200_EXTENSIONS_H_
#define XGB_B200_EXTENSIONS_H_

#include "xgboost/c_api.h"

/* Hex encoding of an NCCL unique id, to be shared with every rank before
 * XGCommunicatorInit. Replaces the tracker of upstream's collective module
 * (python-package/xgboost/collective.py in the reference). */
XGB_DLL int XGBBNcclUniqueId(char const** out);
/* Selects the CUDA device of the calling thread. */
XGB_DLL int XGBBSetDevice(int device);
/* Waits for all work on the current device. */
XGB_DLL int XGBBSynchronize(void);
/* Quantises a matrix now (QuantileDMatrix), with the cuts of `ref` when it is
 * not NULL. Replaces XGQuantileDMatrixCreateFromCallback
 * (include/xgboost/c_api.h:535) for in-memory data. */
XGB_DLL int XGDMatrixQuantise(DMatrixHandle handle, int max_bin, DMatrixHandle ref);
/* JSON {"hist_ms", "hist_bytes", "hist_launches", "rounds"}: CUDA-event time of the
 * histogram kernels when the booster has cuda_profile=1. Replaces
 * XGBoosterMetalProfile (include/metalgb/c_api.h:8-12). */
XGB_DLL int XGBoosterGetCudaProfile(BoosterHandle handle, char const** out);
/* Clears the counters of XGBoosterGetCudaProfile. */
XGB_DLL int XGBoosterResetCudaProfile(BoosterHandle handle);
/* Asks the next boosting round to keep the built int64 histograms of level
 * `depth` (0 = root) of its first tree; -1 cancels. That tree runs without
 * its CUDA graph. The words kept are the ones the reference's histogram
 * kernels write (kernels/boost.metal:700-733, histogram_missing.metal.h:13-60):
 * one (g, h) pair per (built node, feature, bin), bin B the missing bin. */
XGB_DLL int XGBoosterCaptureLevelHistograms(BoosterHandle handle, int depth);
/* The captured level: meta = JSON {"depth", "pairs", "f_lo", "f_hi", "bins1"};
 * hist = [pairs][f_hi - f_lo][bins1][2] int64 (this rank's features, summed
 * over every rank's rows); node_ids[pairs] = the node each histogram belongs
 * to. Valid until the next call on this thread. */
XGB_DLL int XGBoosterGetLevelHistograms(BoosterHandle handle, char const** meta, int64_t const** hist,
                                        uint32_t const** node_ids);
/* Records CUDA event `slot` (0..63) on the booster's stream, and the device
 * time between two recorded events; used to time whole rounds. */
XGB_DLL int XGBoosterRecordEvent(BoosterHandle handle, int slot);
XGB_DLL int XGBoosterEventElapsed(BoosterHandle handle, int a, int b, float* ms);

/* Kernel-level entry points used by the parity tests (host buffers in, host
 * buffers out). */
/* Cuts (cuts[f * min(max_bin, rows) + i]), counts, minima and row-major bins
 * (0xffffffff = missing) of X [rows][cols]: the reference's
 * Matrix::quantize (src/data.cpp:1210-1306). */
XGB_DLL int XGBBQuantizeHost(const float* X, bst_ulong rows, bst_ulong cols, uint32_t max_bin,
                             float* cuts, uint32_t* counts, float* minima, uint32_t* bins);
/* Cuts (cuts[f * min(max_bin, rows) + i]), counts and minima of X [rows][cols]
 * from the host sketch alone, with `threads` workers (0 = all cores): the
 * reference's Matrix::make_quantile_cuts (src/quantile.cpp:22-213). Needs no
 * GPU. */
XGB_DLL int XGBBSketchHost(const float* X, bst_ulong rows, bst_ulong cols, const float* weights,
                           uint32_t max_bin, int threads, float* cuts, uint32_t* counts, float* minima);
/* The same cuts computed on the GPU (the reference's sketch kernels,
 * kernels/quantile.metal.h:19-400, driven as in src/quantile.cpp:22-213):
 * X [rows][cols] and weights (or NULL) are host arrays copied to the device;
 * results land in the host arrays as for XGBBSketchHost, bit for bit. */
XGB_DLL int XGBBSketchDevice(const float* X, bst_ulong rows, bst_ulong cols, const float* weights,
                             uint32_t max_bin, float* cuts, uint32_t* counts, float* minima);
/* No counterpart in the reference (a measurement of this hardware): SM
 * cycles per warp-level shared-memory instruction when `warps` warps of one
 * block per SM each run `iters` passes of 32 feature steps with the histogram
 * kernels' conflict-free addressing. variant 0: red.shared.add.s32, 4 per
 * code; 1: red.shared.add.s32, 1 per code; 2: st.shared.b32, 4 per code;
 * 3: atom.shared.add.u64, 2 per code. */
XGB_DLL int XGBBProbeSharedPipe(int variant, uint32_t warps, uint32_t iters, double* cycles);
/* One evaluation metric of transformed predictions [rows][groups] (the
 * metric side of XGBoosterEvalOneIter, src/metrics.cpp:8-158); weights may
 * be NULL. Needs no GPU. */
XGB_DLL int XGBBMetricHost(char const* name, const float* pred, bst_ulong rows, uint32_t groups,
                           const float* labels, const float* weights, int multiclass, double* out);
/* No counterpart in the reference, which evaluates in one process. The
 * rank-additive form of a mean-type metric (every metric but auc) used when
 * rows are sharded over workers: sums[0] = sum of weight x per-row term,
 * sums[1] = sum of weights over `rows`; XGBBMetricFromSums turns the sums of
 * all workers into the metric (a square root for rmse and rmsle). AUC is
 * refused: it needs all rows. */
XGB_DLL int XGBBMetricSumsHost(char const* name, const float* pred, bst_ulong rows, uint32_t groups,
                               const float* labels, const float* weights, int multiclass, double* sums);
XGB_DLL int XGBBMetricFromSums(char const* name, double loss_sum, double weight_sum, double* out);
/* Gradient pairs [groups][rows][2] and power-of-two scales [groups][2]: the
 * reference's gradients + gradient_partial_sums + gradient_scales
 * (kernels/boost.metal:553-601, kernels/gradient_quantization.metal.h:1-67). */
XGB_DLL int XGBBGradientsHost(int objective, const float* margins, const float* labels,
                              const float* weights, bst_ulong rows, uint32_t groups,
                              float scale_pos_weight, float* pairs, float* scales);
/* No counterpart in the reference. Device-pointer variant of
 * XGBBGradientsHost that allocates no device memory: margins [rows][groups],
 * labels [rows], weights [rows] or NULL, pairs [groups][rows][2] and scales
 * [groups][2] are caller-owned device buffers, and the scale accumulators live
 * in one fixed 17,408-byte device array of the library, cleared on `stream`
 * (a cudaStream_t, NULL = default stream) at the start of every call. Work is
 * enqueued on `stream` and not waited for.
 * Limit: 1 <= groups <= 64 and 1 <= rows < 2^32; other sizes are rejected with
 * an error before anything is enqueued.
 * For callers that cannot allocate: a custom-objective loop stepping beside
 * training on its own stream, where cudaMalloc/cudaFree would synchronise the
 * device and stall the other streams, and a process whose device memory is
 * already claimed by a pool allocator, where a per-call allocation can fail
 * mid-run.
 * Calls that can overlap on one device (different streams or unordered host
 * threads) race on the shared array; calls on one stream are safe. The first
 * call on each device looks up the array's address (cudaGetSymbolAddress) and
 * should come before any stream capture on that device; after a device reset
 * (cudaDeviceReset) the first call looks it up again in the new context, and
 * that call too should come before any capture. */
XGB_DLL int XGBBGradientsDeviceNoAlloc(int objective, const float* margins, const float* labels,
                                       const float* weights, bst_ulong rows, uint32_t groups,
                                       float scale_pos_weight, float* pairs, float* scales,
                                       void* stream);
/* `rounds` rounds of training; trees back to back as 48-byte node records
 * {left, right, parent, feature, split_bin, default_left, threshold, leaf,
 * cover, gain, base_weight, flags}, tree sizes, and the final training
 * margins [rows][groups]. The reference's Learner::update loop
 * (src/learner.cpp:632-985). */
XGB_DLL int XGBBTrainHost(const float* X, bst_ulong rows, bst_ulong cols, const float* labels,
                          const float* weights, char const* params_json, uint32_t rounds,
                          void* nodes, bst_ulong node_capacity, uint32_t* tree_sizes,
                          float* margins);

#endif /* XGB_B200_EXTENSIONS_H_ */
