// pkt's include/dependency.cuh, forwarded to this build's pk/dependency.cuh (pkt programs and tests
// that include "../include/dependency.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/dependency.cuh>
