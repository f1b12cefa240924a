// Tadma.hpp - umbrella header of the static-shape Tensor API (the one header
// generated graph code includes, as the reference's Tadma.hpp:1-4).
// Link with -L<repo>/tadma_b200 -ltadma_b200 (libtadma_b200.so, sm_100a).
#pragma once

#include "Constexpr.hpp"
#include "Core.hpp"
#include "ExecutionTape.hpp"
#include "Lazy.hpp"
#include "Node.hpp"
#include "NodeOps.hpp"
#include "Operations.hpp"
#include "Sequence.hpp"
#include "Tensor.hpp"
