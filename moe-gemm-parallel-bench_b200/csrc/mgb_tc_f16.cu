// Native kernel instances for element type __half.
#define MGB_ELEM __half
#include "mgb_instances.cuh"
