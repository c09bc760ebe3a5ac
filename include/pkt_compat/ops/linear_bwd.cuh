// pkt's include/ops/linear_bwd.cuh, forwarded to this build's pk/ops/linear_bwd.cuh.
#pragma once
#include <pk/ops/linear_bwd.cuh>
