// Target verify attention (tcgen05) -- placeholder until the kernel lands.
#include "attn_common.cuh"

namespace neb {

long long verify_workers(int device) { return num_sms(device); }

int verify_group_rows(int gqa) {
  if (gqa < 1 || gqa > 16) return 0;
  int rows = 64 / gqa;
  return rows < 1 ? 1 : rows;
}

int launch_verify(const AttnParams&, long long, cudaStream_t) {
  return set_error(NEB_ERR_UNSUPPORTED, "verify kernel not built yet");
}

}  // namespace neb
