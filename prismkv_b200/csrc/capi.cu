// Library facts for callers that load the C ABI (prismkv_b200.h).
#include "common.cuh"

extern "C" int pk_version(void) {
    // Target sm version (sm_100a) times 100, plus the ABI revision.
    return 100 * 100 + 1;
}

extern "C" int pk_supported_head_dim(int d) { return d == 128; }
