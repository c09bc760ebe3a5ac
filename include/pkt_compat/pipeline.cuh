// pkt's include/pipeline.cuh, forwarded to this build's pk/pipeline.cuh (pkt programs and tests
// that include "../include/pipeline.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/pipeline.cuh>
