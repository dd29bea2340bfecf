// Stand-in for the header that hxinfer-engine/include/cache/prefix_cache.h:12
// includes but the reference tree does not ship.  PrefixCacheManager only needs
// the LlamaModel declaration from it.
#include "model/llama_model.h"
