// pkt's include/ops/linear_fwd.cuh, forwarded to this build's pk/ops/linear_fwd.cuh.
#pragma once
#include <pk/ops/linear_fwd.cuh>
