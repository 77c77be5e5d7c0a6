// Host stand-in for the tiny-cuda-nn device header that some reference
// renderer headers include: the vector types of vec.h (test infrastructure;
// see there).
#pragma once

#include "common.h"
