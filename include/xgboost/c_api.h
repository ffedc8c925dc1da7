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
