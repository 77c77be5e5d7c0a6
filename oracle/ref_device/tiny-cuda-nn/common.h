// Host stand-in for the tiny-cuda-nn common header the reference's sensor
// header includes: the vector types of vec.h (test infrastructure; see there).
#pragma once

#include <type_traits>

#include "vec.h"
