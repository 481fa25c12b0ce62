// Tensor-core beam step (tcgen05 / TMEM / TMA) -- placeholder until the tile
// kernel lands: every call reports "unsupported" so the row kernel runs.
#include "vtnk_internal.h"

namespace vtnk {

bool tc_enabled() { return false; }

int launch_beam_step_tc(const TcArgs&, cudaStream_t) { return VTNK_ERR_UNSUPPORTED; }

}  // namespace vtnk
