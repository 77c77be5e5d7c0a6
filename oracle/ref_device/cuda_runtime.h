// Stand-in for the CUDA runtime header in the host builds of the reference's
// device headers: the host definitions of cuda_host_shim.h (test
// infrastructure; see there).
#pragma once

#include "cuda_host_shim.h"
