// pkt's include/block_runtime.cuh, forwarded to this build's pk/block_runtime.cuh (pkt programs and tests
// that include "../include/block_runtime.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/block_runtime.cuh>
