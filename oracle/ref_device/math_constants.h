// Stand-in for the CUDA math-constants header in the host builds of the
// reference's device headers (test infrastructure): the infinities they use.
#pragma once

#include <limits>

#define CUDART_INF_F (std::numeric_limits<float>::infinity())
#define CUDART_INF (std::numeric_limits<double>::infinity())
