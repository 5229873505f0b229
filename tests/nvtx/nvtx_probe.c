/*
 * nvtx_probe.c -- a minimal NVTX tool library for the tests.  TEST ONLY.
 *
 * Loaded by the NVTX v3 headers compiled into libpkv_b200.so when the
 * process sets NVTX_INJECTION64_PATH to this library.  It replaces the
 * RangePushA / RangePop slots of the core NVTX module and records the names
 * of the ranges pushed, in order, so a test can read them back with
 * probe_ranges() (names separated by '\n') and probe_depth() (pushes minus
 * pops: 0 when every range was closed).
 */
#include <stdint.h>
#include <string.h>

#include <nvtx3/nvToolsExt.h>

static char g_log[1 << 16];
static size_t g_used;
static int g_depth;

static int probe_push(const char *name) {
    const size_t n = strlen(name);
    if (g_used + n + 2 < sizeof(g_log)) {
        memcpy(g_log + g_used, name, n);
        g_used += n;
        g_log[g_used++] = '\n';
        g_log[g_used] = 0;
    }
    return ++g_depth;
}

static int probe_pop(void) { return --g_depth; }

const char *probe_ranges(void) { return g_log; }
int probe_depth(void) { return g_depth; }

int InitializeInjectionNvtx2(NvtxGetExportTableFunc_t get_table) {
    const NvtxExportTableCallbacks *cb =
        (const NvtxExportTableCallbacks *)get_table(NVTX_ETID_CALLBACKS);
    NvtxFunctionTable table = 0;
    unsigned int size = 0;
    if (cb == 0 || !cb->GetModuleFunctionTable(NVTX_CB_MODULE_CORE, &table, &size) ||
        size <= NVTX_CBID_CORE_RangePop)
        return 0;
    *table[NVTX_CBID_CORE_RangePushA] = (NvtxFunctionPointer)probe_push;
    *table[NVTX_CBID_CORE_RangePop] = (NvtxFunctionPointer)probe_pop;
    return 1;
}
