// Native kernel instances for element type __nv_bfloat16.
#define MGB_ELEM __nv_bfloat16
#include "mgb_instances.cuh"
