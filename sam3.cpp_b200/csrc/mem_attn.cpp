// Memory attention on B200 (host orchestration).
#include "engine.h"

namespace s3b {

int mem_attn_run(s3b_ctx* ctx, const float* curr, const float* src_pos, int feat, const float* prompt,
                 const float* prompt_pos, int m_total, int n_ptr, float* out) {
  (void)curr; (void)src_pos; (void)feat; (void)prompt; (void)prompt_pos; (void)m_total; (void)n_ptr; (void)out;
  return set_error(ctx, kErrUnsupported, "memory attention not built yet");
}

}  // namespace s3b
