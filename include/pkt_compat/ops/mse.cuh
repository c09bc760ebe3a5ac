// pkt's include/ops/mse.cuh, forwarded to this build's pk/ops/mse.cuh.
#pragma once
#include <pk/ops/mse.cuh>
