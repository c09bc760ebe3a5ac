// pkt's include/ops/sgd.cuh, forwarded to this build's pk/ops/sgd.cuh.
#pragma once
#include <pk/ops/sgd.cuh>
