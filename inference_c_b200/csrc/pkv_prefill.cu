// pkv_prefill.cu -- chunked prefill attention over the paged cache (sm_100a).
#include "pkv_device.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {
__device__ uint32_t g_prefill_fault;
}  // namespace
}  // namespace pkv

extern "C" {

int pkv_paged_prefill(const PkvPagedLayer *layer, const PkvBatch *batch, size_t q_heads,
                      const int32_t *query_offsets, const void *query, size_t total_query_rows,
                      size_t max_query_len, float scale, int causal, void *output,
                      PkvDType output_dtype, PkvStream stream, char *error,
                      size_t error_capacity) {
    (void)layer; (void)batch; (void)q_heads; (void)query_offsets; (void)query;
    (void)total_query_rows; (void)max_query_len; (void)scale; (void)causal; (void)output;
    (void)output_dtype; (void)stream;
    pkv_internal_set_error(error, error_capacity, "pkv_paged_prefill: not built yet");
    return 0;
}

int pkv_internal_take_prefill_fault(uint32_t *code) {
    uint32_t zero = 0;
    if (cudaMemcpyFromSymbol(code, pkv::g_prefill_fault, sizeof(uint32_t)) != cudaSuccess) return 0;
    return cudaMemcpyToSymbol(pkv::g_prefill_fault, &zero, sizeof(uint32_t)) == cudaSuccess;
}

}  // extern "C"
