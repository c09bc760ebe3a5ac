// pkt's include/ops/zero.cuh, forwarded to this build's pk/ops/zero.cuh.
#pragma once
#include <pk/ops/zero.cuh>
