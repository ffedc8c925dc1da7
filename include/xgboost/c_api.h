/*
 * C ABI of the B200 histogram tree trainer: the upstream XGBoost entry points
 * on the training and prediction path, with the upstream signatures. Each
 * declaration names the reference interface it replaces (paths inside
 * tabulai/xgboost-metal). Conventions as upstream: every int-returning call
 * gives 0 on success and -1 on failure, with the message available from
 * XGBGetLastError on the same thread (src/c_api.cpp:33-40); pointers returned
 * through out-parameters stay valid until the next call on that thread
 * (src/c_api.cpp:20-29).
 */
#ifndef XGB_B200_XGBOOST_C_API_H_
#define XGB_B200_XGBOOST_C_API_H_

#ifdef __cplusplus
#define XGB_EXTERN_C extern "C"
#include <cstdint>
#else
#define XGB_EXTERN_C
#include <stdint.h>
#endif

#define XGB_DLL XGB_EXTERN_C __attribute__((visibility("default")))

typedef uint64_t bst_ulong;
typedef void* DMatrixHandle;
typedef void* BoosterHandle;
/* include/xgboost/c_api.h:371-474: the caller's batch iterator. */
typedef void* DataIterHandle;
typedef int XGDMatrixCallbackNext(DataIterHandle iter);
typedef void DataIterResetCallback(DataIterHandle handle);

/* include/xgboost/c_api.h:1865-1875: a strided 1-D or 2-D host buffer.
 * dtype_code: 1 f32, 2 f64, 3 f16, 4 bf16, 5 i8, 6 i16, 7 i32, 8 i64, 9 u8,
 * 10 u16, 11 u32, 12 u64, 13 bool bytes, 14 LSB-first bits (one column).
 * flags: bit 0 C-contiguous (strides ignored), bit 1 zero copy preferred,
 * bit 2 strides[0] = first bit of a bit buffer. mask_mode (one entry per
 * row, from mask_bit_offset): 0 none, 1 LSB-first valid bits, 2 nonzero
 * bytes valid, 3 nonzero bytes invalid; invalid rows read as missing. */
typedef struct {
  const void* data;
  uint64_t shape[2];
  int64_t strides[2];
  uint32_t ndim;
  uint32_t dtype_code;
  const void* mask_data;
  int64_t mask_bit_offset;
  uint32_t mask_mode;
  uint32_t flags;
} XGBufferDescriptor;

/* --- library ------------------------------------------------------------ */
/* include/xgboost/c_api.h:68 */
XGB_DLL void XGBoostVersion(int* major, int* minor, int* patch);
/* include/xgboost/c_api.h:77 */
XGB_DLL int XGBuildInfo(char const** out);
/* include/xgboost/c_api.h:90 */
XGB_DLL const char* XGBGetLastError(void);
/* include/xgboost/c_api.h:101 */
XGB_DLL int XGBRegisterLogCallback(void (*callback)(const char*));
/* include/xgboost/c_api.h:111 */
XGB_DLL int XGBSetGlobalConfig(char const* config);
/* include/xgboost/c_api.h:118 */
XGB_DLL int XGBGetGlobalConfig(char const** out_config);

/* --- DMatrix ------------------------------------------------------------- */
/* include/xgboost/c_api.h:240 (src/c_api.cpp:192): dense __array_interface__ JSON;
 * config {"missing": float|null, "nthread": int}. */
XGB_DLL int XGDMatrixCreateFromDense(char const* data, char const* config, DMatrixHandle* out);
/* include/xgboost/c_api.h:273 */
XGB_DLL int XGDMatrixCreateFromMat(const float* data, bst_ulong nrow, bst_ulong ncol, float missing,
                                   DMatrixHandle* out);
/* include/xgboost/c_api.h:221 (src/c_api.cpp:198): CSR; absent entries are missing. */
XGB_DLL int XGDMatrixCreateFromCSR(char const* indptr, char const* indices, char const* data,
                                   bst_ulong ncol, char const* config, DMatrixHandle* out);
/* include/xgboost/c_api.h:666 */
XGB_DLL int XGDMatrixFree(DMatrixHandle handle);
/* include/xgboost/c_api.h:692: fields "label", "weight", "base_margin". */
XGB_DLL int XGDMatrixSetInfoFromInterface(DMatrixHandle handle, char const* field, char const* data);
/* include/xgboost/c_api.h:703 */
XGB_DLL int XGDMatrixSetFloatInfo(DMatrixHandle handle, const char* field, const float* array,
                                  bst_ulong len);
/* include/xgboost/c_api.h:878 */
XGB_DLL int XGDMatrixGetFloatInfo(const DMatrixHandle handle, const char* field, bst_ulong* out_len,
                                  const float** out_dptr);
/* include/xgboost/c_api.h:901 */
XGB_DLL int XGDMatrixNumRow(DMatrixHandle handle, bst_ulong* out);
/* include/xgboost/c_api.h:909 */
XGB_DLL int XGDMatrixNumCol(DMatrixHandle handle, bst_ulong* out);
/* include/xgboost/c_api.h:919 */
XGB_DLL int XGDMatrixNumNonMissing(DMatrixHandle handle, bst_ulong* out);
/* include/xgboost/c_api.h:1877 (src/c_api.cpp:838-844). */
XGB_DLL int XGDMatrixCreateFromBufferDescriptor(XGBufferDescriptor const* desc, float missing,
                                                DMatrixHandle* out);
/* include/xgboost/c_api.h:1881: fields as XGDMatrixSetInfoFromInterface. */
XGB_DLL int XGDMatrixSetInfoFromBufferDescriptor(DMatrixHandle handle, char const* field,
                                                 XGBufferDescriptor const* desc);
/* include/xgboost/c_api.h:460: the batch holder filled by an iterator's next(). */
XGB_DLL int XGProxyDMatrixCreate(DMatrixHandle* out);
/* include/xgboost/c_api.h:622 */
XGB_DLL int XGProxyDMatrixSetDataDense(DMatrixHandle handle, char const* data);
/* include/xgboost/c_api.h:635 */
XGB_DLL int XGProxyDMatrixSetDataCSR(DMatrixHandle handle, char const* indptr, char const* indices,
                                     char const* data, bst_ulong ncol);
/* include/xgboost/c_api.h:499 (src/c_api.cpp:140-157, 222-224): batches
 * concatenated on the host; config {"missing"}. */
XGB_DLL int XGDMatrixCreateFromCallback(DataIterHandle iter, DMatrixHandle proxy,
                                        DataIterResetCallback* reset, XGDMatrixCallbackNext* next,
                                        char const* config, DMatrixHandle* out);
/* include/xgboost/c_api.h:535 (src/c_api.cpp:225-239): as above, then
 * quantised on the GPU with the cuts of `ref` (a DMatrix handle) when given;
 * config {"missing", "max_bin"}. */
XGB_DLL int XGQuantileDMatrixCreateFromCallback(DataIterHandle iter, DMatrixHandle proxy, DataIterHandle ref,
                                                DataIterResetCallback* reset, XGDMatrixCallbackNext* next,
                                                char const* config, DMatrixHandle* out);

/* --- Booster -------------------------------------------------------------- */
/* include/xgboost/c_api.h:996 (src/c_api.cpp:442-452) */
XGB_DLL int XGBoosterCreate(const DMatrixHandle dmats[], bst_ulong len, BoosterHandle* out);
/* include/xgboost/c_api.h:1008 */
XGB_DLL int XGBoosterFree(BoosterHandle handle);
/* include/xgboost/c_api.h:1045 */
XGB_DLL int XGBoosterBoostedRounds(BoosterHandle handle, int* out);
/* include/xgboost/c_api.h:1058: aliases eta, lambda, alpha, gamma as in src/learner.cpp:111-118. */
XGB_DLL int XGBoosterSetParam(BoosterHandle handle, const char* name, const char* value);
/* include/xgboost/c_api.h:1072 */
XGB_DLL int XGBoosterSetParams(BoosterHandle handle, char const* config);
/* include/xgboost/c_api.h:1083 */
XGB_DLL int XGBoosterGetNumFeature(BoosterHandle handle, bst_ulong* out);
/* include/xgboost/c_api.h:1095 (src/c_api.cpp:484): one boosting round on the GPU. */
XGB_DLL int XGBoosterUpdateOneIter(BoosterHandle handle, int iter, DMatrixHandle dtrain);
/* include/xgboost/c_api.h:1134 (src/c_api.cpp:498-500, src/learner.cpp:1025-1048):
 * "[iter]\t<name>-<metric>:<value>" over the given matrices for every
 * eval_metric (rmse, mae, rmsle, mape, logloss, error[@t], merror, mlogloss,
 * auc), or the objective's default metric. */
XGB_DLL int XGBoosterEvalOneIter(BoosterHandle handle, int iter, DMatrixHandle dmats[], const char* evnames[],
                                 bst_ulong len, const char** out_result);
/* include/xgboost/c_api.h:1121 (src/c_api.cpp:485-487): one round from a custom
 * objective; grad and hess are __array_interface__ JSON of shape (rows,) or
 * (rows, groups), finite. Without base_score the intercept is 0.5. */
XGB_DLL int XGBoosterTrainOneIter(BoosterHandle handle, DMatrixHandle dtrain, int iter, char const* grad,
                                  char const* hess);
/* include/xgboost/c_api.h:1103: the same from flat float arrays of len = rows * groups. */
XGB_DLL int XGBoosterBoostOneIter(BoosterHandle handle, DMatrixHandle dtrain, float* grad, float* hess,
                                  bst_ulong len);
/* include/xgboost/c_api.h:1207 (src/c_api.cpp:507): config {"type": 0 value | 1 margin,
 * "training", "iteration_begin", "iteration_end", "strict_shape"}. */
XGB_DLL int XGBoosterPredictFromDMatrix(BoosterHandle handle, DMatrixHandle dmat, char const* config,
                                        bst_ulong const** out_shape, bst_ulong* out_dim,
                                        float const** out_result);
/* Legacy upstream entry named by the task (older XGBoost headers; the
 * reference header has only the c_api.h:1207-1339 predict family): bit 0 of
 * option_mask = margins, ntree_limit = rounds to use (0 = all). */
XGB_DLL int XGBoosterPredict(BoosterHandle handle, DMatrixHandle dmat, int option_mask,
                             unsigned ntree_limit, int training, bst_ulong* out_len,
                             const float** out_result);
/* include/xgboost/c_api.h:1234 (src/c_api.cpp:510-512): in-place prediction
 * from a dense __array_interface__; config as XGBoosterPredictFromDMatrix plus
 * "missing"; base margins from the proxy `m` when not NULL. */
XGB_DLL int XGBoosterPredictFromDense(BoosterHandle handle, char const* values, char const* config,
                                      DMatrixHandle m, bst_ulong const** out_shape, bst_ulong* out_dim,
                                      const float** out_result);
/* include/xgboost/c_api.h:1020: releases the training state; the model stays. */
XGB_DLL int XGBoosterReset(BoosterHandle handle);
/* include/xgboost/c_api.h:1035 (src/c_api.cpp:503-506): rounds begin, begin+step,
 * ... < end (end 0 = all) as a new booster; -2 when out of range. */
XGB_DLL int XGBoosterSlice(BoosterHandle handle, int begin_layer, int end_layer, int step,
                           BoosterHandle* out);
/* include/xgboost/c_api.h:1378. Loads a JSON or UBJSON model file (upstream XGBoost's schema). */
XGB_DLL int XGBoosterLoadModel(BoosterHandle handle, const char* fname);
/* include/xgboost/c_api.h:1387. JSON when the name ends in ".json", else UBJSON. */
XGB_DLL int XGBoosterSaveModel(BoosterHandle handle, const char* fname);
/* include/xgboost/c_api.h:1396. */
XGB_DLL int XGBoosterLoadModelFromBuffer(BoosterHandle handle, const void* buf, bst_ulong len);
/* include/xgboost/c_api.h:1414. config: {"format": "json" | "ubj"} (default "ubj"). */
XGB_DLL int XGBoosterSaveModelToBuffer(BoosterHandle handle, char const* config, bst_ulong* out_len,
                                       char const** out_dptr);
/* include/xgboost/c_api.h:1451 */
XGB_DLL int XGBoosterSaveJsonConfig(BoosterHandle handle, bst_ulong* out_len, char const** out_str);
/* include/xgboost/c_api.h:1461 (src/model.cpp:287-333). */
XGB_DLL int XGBoosterLoadJsonConfig(BoosterHandle handle, char const* config);
/* include/xgboost/c_api.h:1426: {"Config", "Model"} as UBJSON (pickling). */
XGB_DLL int XGBoosterSerializeToBuffer(BoosterHandle handle, bst_ulong* out_len, char const** out_dptr);
/* include/xgboost/c_api.h:1437 */
XGB_DLL int XGBoosterUnserializeFromBuffer(BoosterHandle handle, const void* buf, bst_ulong len);
/* include/xgboost/c_api.h:1473: text dump. */
XGB_DLL int XGBoosterDumpModel(BoosterHandle handle, const char* fmap, int with_stats, bst_ulong* out_len,
                               const char*** out_dump_array);
/* include/xgboost/c_api.h:1486 (src/model.cpp:334-429): format "text", "json"
 * or "dot"; fmap must be empty. */
XGB_DLL int XGBoosterDumpModelEx(BoosterHandle handle, const char* fmap, int with_stats, const char* format,
                                 bst_ulong* out_len, const char*** out_dump_array);
/* include/xgboost/c_api.h:1501 */
XGB_DLL int XGBoosterDumpModelWithFeatures(BoosterHandle handle, int fnum, const char** fname,
                                           const char** ftype, int with_stats, bst_ulong* out_len,
                                           const char*** out_models);
/* include/xgboost/c_api.h:1517 */
XGB_DLL int XGBoosterDumpModelExWithFeatures(BoosterHandle handle, int fnum, const char** fname,
                                             const char** ftype, int with_stats, const char* format,
                                             bst_ulong* out_len, const char*** out_models);
/* include/xgboost/c_api.h:1633 (src/c_api.cpp:590-620): config
 * {"importance_type", "feature_names"}; features used by a split only. */
XGB_DLL int XGBoosterFeatureScore(BoosterHandle handle, const char* config, bst_ulong* out_n_features,
                                  char const*** out_features, bst_ulong* out_dim,
                                  bst_ulong const** out_shape, float const** out_scores);
/* include/xgboost/c_api.h:1548 */
XGB_DLL int XGBoosterGetAttr(BoosterHandle handle, const char* key, const char** out, int* success);
/* include/xgboost/c_api.h:1558 */
XGB_DLL int XGBoosterSetAttr(BoosterHandle handle, const char* key, const char* value);
/* include/xgboost/c_api.h:1566 */
XGB_DLL int XGBoosterGetAttrNames(BoosterHandle handle, bst_ulong* out_len, const char*** out);
/* include/xgboost/c_api.h:1583 */
XGB_DLL int XGBoosterSetStrFeatureInfo(BoosterHandle handle, const char* field, const char** features,
                                       const bst_ulong size);
/* include/xgboost/c_api.h:1605 */
XGB_DLL int XGBoosterGetStrFeatureInfo(BoosterHandle handle, const char* field, bst_ulong* len,
                                       const char*** out_features);

/* --- collective ----------------------------------------------------------- */
/* include/xgboost/c_api.h:1768 (a stub in the reference, src/c_api.cpp:600-614):
 * config {"rank", "world_size", "device", "nccl_unique_id"}; world_size > 1
 * shards rows over one NCCL communicator per process. */
XGB_DLL int XGCommunicatorInit(char const* config);
/* include/xgboost/c_api.h:1777 */
XGB_DLL int XGCommunicatorFinalize(void);
/* upstream include/xgboost/c_api.h XGCommunicatorGetRank / GetWorldSize */
XGB_DLL int XGCommunicatorGetRank(void);
XGB_DLL int XGCommunicatorGetWorldSize(void);

#endif /* XGB_B200_XGBOOST_C_API_H_ */
