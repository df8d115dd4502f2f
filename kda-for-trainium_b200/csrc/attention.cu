// Grouped-query attention (placeholder until the tcgen05 attention kernel lands).
#include "common.cuh"

extern "C" kda_status kda_gqa_full_bf16(const void* q, const void* k, const void* v, void* out, int64_t B, int64_t S,
                                        int64_t QH, int64_t KH, int64_t D, int causal, float rope_theta, int out_bshd,
                                        void* stream) {
  (void)causal; (void)rope_theta; (void)out_bshd; (void)stream;
  KDA_CHECK_ARG(q && k && v && out, "gqa_full: null pointer");
  KDA_CHECK_ARG(B > 0 && S > 0 && QH > 0 && KH > 0 && QH % KH == 0, "gqa_full: bad sizes");
  KDA_CHECK_SUPPORTED(false, "gqa_full: not implemented yet");
  return KDA_UNSUPPORTED;
}
