// pkt's include/profile_ranges.cuh, forwarded to this build's pk/profile_ranges.cuh (pkt programs and tests
// that include "../include/profile_ranges.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/profile_ranges.cuh>
