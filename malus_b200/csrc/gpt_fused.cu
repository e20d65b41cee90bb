// The fused B200 nanoGPT step (mode 1).  Placeholder until implemented.
#include "common.cuh"
#include <vector>
namespace malus {
struct FusedStep {};
FusedStep* fused_create(const malus_gpt_config&, const std::vector<float*>&, const std::vector<size_t>&,
                        float*, const std::vector<size_t>&) {
  panic("fused nanoGPT step (mode 1) is not built yet");
}
void fused_destroy(FusedStep* f) { delete f; }
void fused_step(FusedStep*, const int32_t*, const int32_t*, float*) { panic("fused step unavailable"); }
}  // namespace malus
