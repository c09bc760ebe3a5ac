// pkt's include/perf_counters.cuh, forwarded to this build's pk/perf_counters.cuh (pkt programs and tests
// that include "../include/perf_counters.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/perf_counters.cuh>
