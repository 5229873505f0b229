/*
 * sdk_test_glue.c -- link glue for the SDK's tests/test_attention.c built
 * unchanged against libpkv_b200.so.  TEST INFRASTRUCTURE ONLY.
 *
 * In that binary two libraries keep decoder caches: the SDK's CUDA backend
 * (its contiguous decoders) and libpkv_b200.so (the paged decoder).  The
 * test calls tensor_attention_decode_cache_clear() before each decoder run
 * and expects every cache to be dropped.  The SDK's own function (attention.c,
 * which dispatches to its backend) is renamed in its object file to
 * sdk_tensor_attention_decode_cache_clear; this definition calls it and then
 * libpkv_b200.so's definition, found as the next one in load order.
 */
#define _GNU_SOURCE
#include <dlfcn.h>

void sdk_tensor_attention_decode_cache_clear(void);

void tensor_attention_decode_cache_clear(void) {
    sdk_tensor_attention_decode_cache_clear();
    void (*paged_clear)(void) =
        (void (*)(void))dlsym(RTLD_NEXT, "tensor_attention_decode_cache_clear");
    if (paged_clear != 0) paged_clear();
}
