// pkt's include/ops/axpy.cuh, forwarded to this build's pk/ops/axpy.cuh.
#pragma once
#include <pk/ops/axpy.cuh>
