// Reserved translation unit for specialised collective kernels.
#include "vb/launch.h"
