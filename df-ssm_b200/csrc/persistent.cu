// Persistent whole-step decode kernel (small batch): not yet built in this revision.
#include "engine.h"

int persistent_init(dfssm_engine*) { return DFSSM_OK; }
bool persistent_supported(const dfssm_engine*) { return false; }
int launch_persistent_step(dfssm_engine*, cudaStream_t) {
  return dfssm_fail(DFSSM_ERR_UNSUPPORTED, "persistent step kernel not built");
}
