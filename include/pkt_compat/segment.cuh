// pkt's include/segment.cuh, forwarded to this build's pk/segment.cuh (pkt programs and tests
// that include "../include/segment.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/segment.cuh>
