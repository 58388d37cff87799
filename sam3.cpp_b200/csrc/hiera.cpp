// SAM 2.x Hiera image encoder + FPN neck on B200 (host orchestration).
#include "engine.h"

namespace s3b {

int hiera_encode(s3b_ctx* ctx, const float* d_chw, int n_frames, int flags) {
  (void)d_chw;
  (void)n_frames;
  (void)flags;
  return set_error(ctx, kErrUnsupported, "Hiera encoder not built yet");
}

}  // namespace s3b
