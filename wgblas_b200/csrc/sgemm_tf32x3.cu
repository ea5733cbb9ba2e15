// 3xTF32 tensor-core sgemm (tcgen05 + TMEM + TMA) — placeholder until the kernel lands.
#include "internal.h"

size_t wg_tf32x3_workspace_bytes(int64_t, int64_t, int64_t) { return 0; }
bool wg_tf32x3_supported(const wg_device *, int64_t, int64_t, int64_t) { return false; }
wg_status wg_sgemm_tf32x3(wg_device *, int, int, int64_t, int64_t, int64_t, float, const float *, int64_t,
                          const float *, int64_t, float, float *, int64_t, void *) {
  return wg_fail(WG_ERR_NOT_SUPPORTED, "3xTF32 kernel not built");
}
