// Umbrella header for the lrrt C++ layer (light-rocm-runtime include/lrrt/lrrt.hpp).
#ifndef LRRT_LRRT_HPP_
#define LRRT_LRRT_HPP_

#include "lrrt/error.hpp"
#include "lrrt/launch.hpp"
#include "lrrt/memory.hpp"
#include "lrrt/module.hpp"
#include "lrrt/runtime.hpp"

#endif // LRRT_LRRT_HPP_
