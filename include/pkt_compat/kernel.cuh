// pkt's include/kernel.cuh, forwarded to this build's pk/kernel.cuh (pkt programs and tests
// that include "../include/kernel.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/kernel.cuh>
