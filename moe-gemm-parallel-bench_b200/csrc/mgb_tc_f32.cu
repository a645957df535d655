// Native kernel instances for element type float.
#define MGB_ELEM float
#include "mgb_instances.cuh"
