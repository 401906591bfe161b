// Umbrella header of the Persistent Graph host API
// (light-rocm-runtime include/lrrt/persistent_graph.hpp).
#ifndef LRRT_PERSISTENT_GRAPH_HPP_
#define LRRT_PERSISTENT_GRAPH_HPP_

#include "lrrt/persistent_graph/abi.hpp"
#include "lrrt/persistent_graph/resident_executor.hpp"

#endif // LRRT_PERSISTENT_GRAPH_HPP_
