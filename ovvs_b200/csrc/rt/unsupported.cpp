// Entry points of the ovvs ABI outside this library's scope (IVF-PQ / RaBitQ, graph indexes, quantizers,
// PCA, SLINK/spectral). They exist so that binaries and bindings built
// against the reference ABI still link and load; each returns OVVS_STATUS_UNSUPPORTED (Destroy
// functions accept any handle, as none can have been created, and return OVVS_STATUS_SUCCESS).
#include "ovvs/ovvs.h"

extern "C" {

ovvsStatus ovvsIvfPqBuild(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric, int32_t nlist, int32_t pq_m, int32_t pq_nbits, ovvsIvfPqIndex_t* index) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)metric; (void)nlist; (void)pq_m; (void)pq_nbits; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfPqSearch(ovvsResources_t res, ovvsIvfPqIndex_t index, const float* queries, int64_t nq, int64_t k, int32_t nprobe, int32_t krefine, const uint8_t* bitset, int64_t* neighbors, float* distances) {
  (void)res; (void)index; (void)queries; (void)nq; (void)k; (void)nprobe; (void)krefine; (void)bitset; (void)neighbors; (void)distances;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfPqSerialize(ovvsIvfPqIndex_t index, const char* path) {
  (void)index; (void)path;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfPqDeserialize(ovvsResources_t res, const char* path, ovvsIvfPqIndex_t* index) {
  (void)res; (void)path; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfPqExtend(ovvsResources_t res, ovvsIvfPqIndex_t index, const float* extra, int64_t nextra) {
  (void)res; (void)index; (void)extra; (void)nextra;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfPqDestroy(ovvsIvfPqIndex_t index) {
  (void)index;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsIvfRabitqBuild(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric, int32_t nlist, ovvsIvfRabitqIndex_t* index) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)metric; (void)nlist; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfRabitqSearch(ovvsResources_t res, ovvsIvfRabitqIndex_t index, const float* queries, int64_t nq, int64_t k, int32_t nprobe, int32_t krefine, const uint8_t* bitset, int64_t* neighbors, float* distances) {
  (void)res; (void)index; (void)queries; (void)nq; (void)k; (void)nprobe; (void)krefine; (void)bitset; (void)neighbors; (void)distances;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfRabitqSerialize(ovvsIvfRabitqIndex_t index, const char* path) {
  (void)index; (void)path;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfRabitqDeserialize(ovvsResources_t res, const char* path, ovvsIvfRabitqIndex_t* index) {
  (void)res; (void)path; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfRabitqExtend(ovvsResources_t res, ovvsIvfRabitqIndex_t index, const float* extra, int64_t nextra) {
  (void)res; (void)index; (void)extra; (void)nextra;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsIvfRabitqDestroy(ovvsIvfRabitqIndex_t index) {
  (void)index;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsNnDescentBuild(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric, int32_t graph_degree, int32_t iterations, ovvsNnDescentGraph_t* graph) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)metric; (void)graph_degree; (void)iterations; (void)graph;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsNnDescentNeighbors(ovvsNnDescentGraph_t graph, const int32_t** ids, int64_t* n, int32_t* degree) {
  (void)graph; (void)ids; (void)n; (void)degree;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsNnDescentDestroy(ovvsNnDescentGraph_t graph) {
  (void)graph;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsCagraBuild(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric, int32_t graph_degree, int32_t intermediate_degree, ovvsCagraIndex_t* index) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)metric; (void)graph_degree; (void)intermediate_degree; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraBuildEx(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric, int32_t graph_degree, int32_t intermediate_degree, ovvsCagraBuildAlgo algo, ovvsCagraIndex_t* index) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)metric; (void)graph_degree; (void)intermediate_degree; (void)algo; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraBuildEx2(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric, int32_t graph_degree, int32_t intermediate_degree, ovvsCagraBuildAlgo algo, ovvsCagraStorage storage, ovvsCagraIndex_t* index) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)metric; (void)graph_degree; (void)intermediate_degree; (void)algo; (void)storage; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraSearch(ovvsResources_t res, ovvsCagraIndex_t index, const float* queries, int64_t nq, int64_t k, int32_t itopk_size, int32_t search_width, const uint8_t* bitset, int64_t* neighbors, float* distances) {
  (void)res; (void)index; (void)queries; (void)nq; (void)k; (void)itopk_size; (void)search_width; (void)bitset; (void)neighbors; (void)distances;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraWalOpen(ovvsResources_t res, ovvsCagraIndex_t index, const char* path, int32_t fsync_every) {
  (void)res; (void)index; (void)path; (void)fsync_every;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraWalClose(ovvsCagraIndex_t index) {
  (void)index;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsCagraCalibrate(ovvsResources_t res, ovvsCagraIndex_t index, float target_recall, int64_t k, int32_t* itopk, int32_t* width, float* achieved) {
  (void)res; (void)index; (void)target_recall; (void)k; (void)itopk; (void)width; (void)achieved;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraQuantize(ovvsResources_t res, ovvsCagraIndex_t index, int32_t pq_m, int32_t pq_nbits) {
  (void)res; (void)index; (void)pq_m; (void)pq_nbits;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraDetachDataset(ovvsCagraIndex_t index) {
  (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraAttachDataset(ovvsCagraIndex_t index, const float* dataset, int64_t n, int64_t dim) {
  (void)index; (void)dataset; (void)n; (void)dim;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraSerialize(ovvsCagraIndex_t index, const char* path) {
  (void)index; (void)path;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraSerializeEx(ovvsCagraIndex_t index, const char* path, int32_t include_dataset) {
  (void)index; (void)path; (void)include_dataset;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraDeserialize(ovvsResources_t res, const char* path, ovvsCagraIndex_t* index) {
  (void)res; (void)path; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraExtend(ovvsResources_t res, ovvsCagraIndex_t index, const float* extra, int64_t nextra) {
  (void)res; (void)index; (void)extra; (void)nextra;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraExtendEx(ovvsResources_t res, ovvsCagraIndex_t index, const float* extra, int64_t nextra, int64_t* out_ids) {
  (void)res; (void)index; (void)extra; (void)nextra; (void)out_ids;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraDelete(ovvsResources_t res, ovvsCagraIndex_t index, const int64_t* ids, int64_t nids) {
  (void)res; (void)index; (void)ids; (void)nids;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraUpdate(ovvsResources_t res, ovvsCagraIndex_t index, const int64_t* ids, const float* vectors, int64_t nids) {
  (void)res; (void)index; (void)ids; (void)vectors; (void)nids;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraCounts(ovvsCagraIndex_t index, int64_t* live, int64_t* deleted) {
  (void)index; (void)live; (void)deleted;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsCagraDestroy(ovvsCagraIndex_t index) {
  (void)index;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsHnswFromCagra(ovvsResources_t res, ovvsCagraIndex_t cagra, ovvsHnswIndex_t* index) {
  (void)res; (void)cagra; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsHnswSearch(ovvsResources_t res, ovvsHnswIndex_t index, const float* queries, int64_t nq, int64_t k, int32_t ef, int64_t* neighbors, float* distances) {
  (void)res; (void)index; (void)queries; (void)nq; (void)k; (void)ef; (void)neighbors; (void)distances;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsHnswSerialize(ovvsHnswIndex_t index, const char* path) {
  (void)index; (void)path;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsHnswDeserialize(ovvsResources_t res, const char* path, ovvsHnswIndex_t* index) {
  (void)res; (void)path; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsHnswDestroy(ovvsHnswIndex_t index) {
  (void)index;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsVamanaBuild(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric, int32_t graph_degree, float alpha, ovvsVamanaIndex_t* index) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)metric; (void)graph_degree; (void)alpha; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsVamanaSearch(ovvsResources_t res, ovvsVamanaIndex_t index, const float* queries, int64_t nq, int64_t k, int32_t beam, const uint8_t* bitset, int64_t* neighbors, float* distances) {
  (void)res; (void)index; (void)queries; (void)nq; (void)k; (void)beam; (void)bitset; (void)neighbors; (void)distances;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsVamanaSerialize(ovvsVamanaIndex_t index, const char* path) {
  (void)index; (void)path;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsVamanaDeserialize(ovvsResources_t res, const char* path, ovvsVamanaIndex_t* index) {
  (void)res; (void)path; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsVamanaMmap(ovvsResources_t res, const char* path, ovvsVamanaIndex_t* index) {
  (void)res; (void)path; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsVamanaDestroy(ovvsVamanaIndex_t index) {
  (void)index;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsScannBuild(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric, int32_t nlist, int32_t pq_m, ovvsScannIndex_t* index) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)metric; (void)nlist; (void)pq_m; (void)index;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsScannSearch(ovvsResources_t res, ovvsScannIndex_t index, const float* queries, int64_t nq, int64_t k, int32_t nprobe, int32_t krefine, int64_t* neighbors, float* distances) {
  (void)res; (void)index; (void)queries; (void)nq; (void)k; (void)nprobe; (void)krefine; (void)neighbors; (void)distances;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsScannDestroy(ovvsScannIndex_t index) {
  (void)index;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsSlinkFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, int32_t nclusters, int32_t knn, ovvsSlinkModel_t* model) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)nclusters; (void)knn; (void)model;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSlinkLabels(ovvsSlinkModel_t model, const int64_t** labels, int64_t* n) {
  (void)model; (void)labels; (void)n;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSlinkDestroy(ovvsSlinkModel_t model) {
  (void)model;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsSpectralFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, int32_t nclusters, int32_t knn, ovvsSpectralModel_t* model) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)nclusters; (void)knn; (void)model;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSpectralLabels(ovvsSpectralModel_t model, const int64_t** labels, int64_t* n) {
  (void)model; (void)labels; (void)n;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSpectralDestroy(ovvsSpectralModel_t model) {
  (void)model;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsSqFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsSqModel_t* model) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)model;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSqEncode(ovvsSqModel_t model, const float* x, int64_t n, uint8_t* codes) {
  (void)model; (void)x; (void)n; (void)codes;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSqDecode(ovvsSqModel_t model, const uint8_t* codes, int64_t n, float* x) {
  (void)model; (void)codes; (void)n; (void)x;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSqDestroy(ovvsSqModel_t model) {
  (void)model;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsPqFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, int32_t pq_m, int32_t pq_nbits, ovvsPqModel_t* model) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)pq_m; (void)pq_nbits; (void)model;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsPqEncode(ovvsPqModel_t model, const float* x, int64_t n, uint8_t* codes) {
  (void)model; (void)x; (void)n; (void)codes;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsPqDecode(ovvsPqModel_t model, const uint8_t* codes, int64_t n, float* x) {
  (void)model; (void)codes; (void)n; (void)x;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsPqDestroy(ovvsPqModel_t model) {
  (void)model;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsBinaryFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, ovvsBinaryQuantizer_t* model) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)model;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsBinaryEncode(ovvsBinaryQuantizer_t model, const float* x, int64_t n, uint8_t* codes) {
  (void)model; (void)x; (void)n; (void)codes;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsBinaryDestroy(ovvsBinaryQuantizer_t model) {
  (void)model;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsPcaFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, int32_t ncomp, ovvsPcaModel_t* model) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)ncomp; (void)model;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsPcaTransform(ovvsPcaModel_t model, const float* x, int64_t n, float* out) {
  (void)model; (void)x; (void)n; (void)out;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsPcaDestroy(ovvsPcaModel_t model) {
  (void)model;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsSpectralEmbedFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim, int32_t ncomp, int32_t knn, ovvsSpectralEmbed_t* model) {
  (void)res; (void)dataset; (void)n; (void)dim; (void)ncomp; (void)knn; (void)model;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSpectralEmbedData(ovvsSpectralEmbed_t model, const float** data, int64_t* n, int32_t* ncomp) {
  (void)model; (void)data; (void)n; (void)ncomp;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsSpectralEmbedDestroy(ovvsSpectralEmbed_t model) {
  (void)model;
  return OVVS_STATUS_SUCCESS;
}

}  // extern "C"
