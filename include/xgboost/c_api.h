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
#include <cstddef>
#include <cstdint>
#else
#define XGB_EXTERN_C
#include <stddef.h>
#include <stdint.h>
#endif

#define XGB_DLL XGB_EXTERN_C __attribute__((visibility("default")))

typedef uint64_t bst_ulong;
typedef void* DMatrixHandle;
typedef void* BoosterHandle;
/* include/xgboost/c_api.h:371-474: the caller's batch iterator. */
typedef void* DataIterHandle;
/* include/xgboost/c_api.h:373-420: the JVM packages' batch iterator. */
typedef void* DataHolderHandle;
typedef struct {
  size_t size;      /* rows in the batch */
  size_t columns;   /* columns of the batch */
  int64_t* offset;  /* size + 1 row offsets */
  float* label;     /* size labels, or NULL */
  float* weight;    /* size weights, or NULL */
  int* index;       /* feature indices */
  float* value;     /* feature values */
} XGBoostBatchCSR;
typedef int XGBCallbackSetData(DataHolderHandle handle, XGBoostBatchCSR batch);
typedef int XGBCallbackDataIterNext(DataIterHandle data_handle, XGBCallbackSetData* set_function,
                                    DataHolderHandle set_function_handle);
/* include/xgboost/c_api.h:57, 1671 */
typedef void* CategoriesHandle;
typedef void* TrackerHandle;
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
/* include/xgboost/c_api.h:254 (src/c_api.cpp:201): CSC; nrow 0 = from indices. */
XGB_DLL int XGDMatrixCreateFromCSC(char const* indptr, char const* indices, char const* data, bst_ulong nrow,
                                   char const* config, DMatrixHandle* out);
/* include/xgboost/c_api.h:260 */
XGB_DLL int XGDMatrixCreateFromCOO(char const* row_idx, char const* col_idx, char const* data, bst_ulong nrow,
                                   bst_ulong ncol, char const* config, DMatrixHandle* out);
/* include/xgboost/c_api.h:205: a JSON list of column array interfaces. */
XGB_DLL int XGDMatrixCreateFromColumnar(char const* data, char const* config, DMatrixHandle* out);
/* include/xgboost/c_api.h:1879 */
XGB_DLL int XGDMatrixCreateFromColumnarBuffers(XGBufferDescriptor const* columns, bst_ulong ncol, float missing,
                                               DMatrixHandle* out);
/* include/xgboost/c_api.h:285 */
XGB_DLL int XGDMatrixCreateFromMat_omp(const float* data, bst_ulong nrow, bst_ulong ncol, float missing,
                                       DMatrixHandle* out, int nthread);
/* include/xgboost/c_api.h:314, 300: device arrays, copied to the host. */
XGB_DLL int XGDMatrixCreateFromCudaArrayInterface(char const* data, char const* config, DMatrixHandle* out);
XGB_DLL int XGDMatrixCreateFromCudaColumnar(char const* data, char const* config, DMatrixHandle* out);
/* include/xgboost/c_api.h:1883 (src/c_api.cpp:872-930): a 2-D DLPack tensor on the
 * host or a CUDA device; its deleter runs before the call returns. */
XGB_DLL int XGDMatrixCreateFromDLPack(void* dl_managed_tensor, int is_versioned, float missing,
                                      DMatrixHandle* out);
/* include/xgboost/c_api.h:1885 (src/c_api.cpp:930-983): an Arrow C-data struct of
 * primitive columns (or one column); schema and array are released. */
XGB_DLL int XGDMatrixCreateFromArrow(void const* arrow_schema, void const* arrow_array, float missing,
                                     DMatrixHandle* out);
/* include/xgboost/c_api.h:431: CSR batches from the legacy iterator. */
XGB_DLL int XGDMatrixCreateFromDataIter(DataIterHandle data_handle, XGBCallbackDataIterNext* callback,
                                        const char* cache_info, float missing, DMatrixHandle* out);
/* include/xgboost/c_api.h:149 (src/c_api.cpp:364-438): {"uri": "path?format=csv"
 * (label_column=K) or "path?format=libsvm"}. */
XGB_DLL int XGDMatrixCreateFromURI(char const* config, DMatrixHandle* out);
/* include/xgboost/c_api.h:681: not implemented (returns -1). */
XGB_DLL int XGDMatrixSaveBinary(DMatrixHandle handle, const char* fname, int silent);
/* include/xgboost/c_api.h:849: type 1 f32, 2 f64, 3 u32, 4 u64. */
XGB_DLL int XGDMatrixSetDenseInfo(DMatrixHandle handle, const char* field, void const* data, bst_ulong size,
                                  int type);
/* include/xgboost/c_api.h:710 */
XGB_DLL int XGDMatrixSetUIntInfo(DMatrixHandle handle, const char* field, const unsigned* array, bst_ulong len);
/* include/xgboost/c_api.h:892: "group_ptr", always empty. */
XGB_DLL int XGDMatrixGetUIntInfo(const DMatrixHandle handle, const char* field, bst_ulong* out_len,
                                 const unsigned** out_dptr);
/* include/xgboost/c_api.h:868: array interface of the matrix's own metadata. */
XGB_DLL int XGDMatrixGetInfoRef(DMatrixHandle handle, char const* field, char const** out_array);
/* include/xgboost/c_api.h:739, 777: "feature_name" / "feature_type". */
XGB_DLL int XGDMatrixSetStrFeatureInfo(DMatrixHandle handle, const char* field, const char** features,
                                       const bst_ulong size);
XGB_DLL int XGDMatrixGetStrFeatureInfo(DMatrixHandle handle, const char* field, bst_ulong* size,
                                       const char*** out_features);
/* include/xgboost/c_api.h:929 */
XGB_DLL int XGDMatrixDataSplitMode(DMatrixHandle handle, bst_ulong* out);
/* include/xgboost/c_api.h:1897 */
XGB_DLL int XGDMatrixWasZeroCopied(DMatrixHandle handle, int* out);
/* include/xgboost/c_api.h:951 */
XGB_DLL int XGDMatrixGetDataAsCSR(DMatrixHandle const handle, char const* config, bst_ulong* out_indptr,
                                  unsigned* out_indices, float* out_data);
/* include/xgboost/c_api.h:969: per feature -inf then its cuts (array interfaces). */
XGB_DLL int XGDMatrixGetQuantileCut(DMatrixHandle const handle, char const* config, char const** out_indptr,
                                    char const** out_data);
/* include/xgboost/c_api.h:648, 659 */
XGB_DLL int XGDMatrixSliceDMatrix(DMatrixHandle handle, const int* idxset, bst_ulong len, DMatrixHandle* out);
XGB_DLL int XGDMatrixSliceDMatrixEx(DMatrixHandle handle, const int* idxset, bst_ulong len, DMatrixHandle* out,
                                    int allow_groups);
/* include/xgboost/c_api.h:1894 (src/c_api.cpp:1017-1117): nfold train/test pairs. */
XGB_DLL int XGDMatrixBuildCVFolds(DMatrixHandle handle, int nfold, unsigned seed, int shuffle, int stratified,
                                  DMatrixHandle* out_train, DMatrixHandle* out_test);
/* include/xgboost/c_api.h:810-842: numerical splits only, so the handle is NULL. */
XGB_DLL int XGDMatrixGetCategories(DMatrixHandle handle, char const* config, CategoriesHandle* out);
XGB_DLL int XGDMatrixGetCategoriesExportToArrow(DMatrixHandle handle, char const* config, CategoriesHandle* out,
                                                char const** export_out);
XGB_DLL int XGBoosterGetCategories(BoosterHandle handle, char const* config, CategoriesHandle* out);
XGB_DLL int XGBoosterGetCategoriesExportToArrow(BoosterHandle handle, char const* config, CategoriesHandle* out,
                                                char const** export_out);
XGB_DLL int XGBCategoriesFree(CategoriesHandle handle);
/* include/xgboost/c_api.h:460: the batch holder filled by an iterator's next(). */
XGB_DLL int XGProxyDMatrixCreate(DMatrixHandle* out);
/* include/xgboost/c_api.h:622 */
XGB_DLL int XGProxyDMatrixSetDataDense(DMatrixHandle handle, char const* data);
/* include/xgboost/c_api.h:635 */
XGB_DLL int XGProxyDMatrixSetDataCSR(DMatrixHandle handle, char const* indptr, char const* indices,
                                     char const* data, bst_ulong ncol);
/* include/xgboost/c_api.h:601, 591, 611 */
XGB_DLL int XGProxyDMatrixSetDataColumnar(DMatrixHandle handle, char const* data);
XGB_DLL int XGProxyDMatrixSetDataCudaArrayInterface(DMatrixHandle handle, const char* data);
XGB_DLL int XGProxyDMatrixSetDataCudaColumnar(DMatrixHandle handle, const char* data);
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
/* include/xgboost/c_api.h:576: in host memory, as the callback QuantileDMatrix. */
XGB_DLL int XGExtMemQuantileDMatrixCreateFromCallback(DataIterHandle iter, DMatrixHandle proxy,
                                                      DataIterHandle ref, DataIterResetCallback* reset,
                                                      XGDMatrixCallbackNext* next, char const* config,
                                                      DMatrixHandle* out);

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
/* include/xgboost/c_api.h:1289, 1261, 1313, 1337, 1887: in-place prediction from
 * CSR, columnar, CUDA and buffer-descriptor inputs (config as PredictFromDense). */
XGB_DLL int XGBoosterPredictFromCSR(BoosterHandle handle, char const* indptr, char const* indices,
                                    char const* values, bst_ulong ncol, char const* config, DMatrixHandle m,
                                    bst_ulong const** out_shape, bst_ulong* out_dim, const float** out_result);
XGB_DLL int XGBoosterPredictFromColumnar(BoosterHandle handle, char const* values, char const* config,
                                         DMatrixHandle m, bst_ulong const** out_shape, bst_ulong* out_dim,
                                         const float** out_result);
XGB_DLL int XGBoosterPredictFromCudaArray(BoosterHandle handle, char const* values, char const* config,
                                          DMatrixHandle proxy, bst_ulong const** out_shape, bst_ulong* out_dim,
                                          const float** out_result);
XGB_DLL int XGBoosterPredictFromCudaColumnar(BoosterHandle handle, char const* data, char const* config,
                                             DMatrixHandle proxy, bst_ulong const** out_shape, bst_ulong* out_dim,
                                             const float** out_result);
XGB_DLL int XGBoosterPredictFromBufferDescriptor(BoosterHandle handle, XGBufferDescriptor const* desc,
                                                 char const* config, DMatrixHandle proxy,
                                                 bst_ulong const** out_shape, bst_ulong* out_dim,
                                                 float const** out_result);
/* include/xgboost/c_api.h:1891 (src/c_api.cpp:1000-1016): into the caller's buffer. */
XGB_DLL int XGBoosterPredictToBuffer(BoosterHandle handle, DMatrixHandle dmat, char const* config,
                                     float* out_buffer, bst_ulong out_capacity, bst_ulong const** out_shape,
                                     bst_ulong* out_dim);
/* include/metalgb/c_api.h:17: vector-leaf trees are not grown (returns -1). */
XGB_DLL int XGBoosterTrainOneIterWithSplitGrad(BoosterHandle handle, DMatrixHandle dtrain, int iter,
                                               char const* grad, char const* hess, char const* value_grad,
                                               char const* value_hess);
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
/* include/xgboost/c_api.h:1798-1858: host buffers over the NCCL communicator;
 * no-ops on one rank. */
XGB_DLL int XGCommunicatorIsDistributed(void);
XGB_DLL int XGCommunicatorPrint(char const* message);
XGB_DLL int XGCommunicatorGetProcessorName(const char** name_str);
XGB_DLL int XGCommunicatorBroadcast(void* send_receive_buffer, size_t size, int root);
XGB_DLL int XGCommunicatorAllreduce(void* send_receive_buffer, size_t count, int data_type, int op);
/* include/metalgb/c_api.h:20: aborts this rank's communicator. */
XGB_DLL int XGCommunicatorSignalError(void);
/* include/xgboost/c_api.h:1697-1742: ranks bootstrap NCCL from a shared unique id
 * instead; these return -1 with that explanation. */
XGB_DLL int XGTrackerCreate(char const* config, TrackerHandle* handle);
XGB_DLL int XGTrackerWorkerArgs(TrackerHandle handle, char const** args);
XGB_DLL int XGTrackerRun(TrackerHandle handle, char const* config);
XGB_DLL int XGTrackerWaitFor(TrackerHandle handle, char const* config);
XGB_DLL int XGTrackerFree(TrackerHandle handle);
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
