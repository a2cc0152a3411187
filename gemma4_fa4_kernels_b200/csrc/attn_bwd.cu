// placeholder until the backward kernels land
#include "../../include/gemma4_b200.h"
extern "C" int g4_attn_bwd(const g4_attn_args*, void*) { return G4_ERR_UNSUPPORTED; }
