// pkt's include/config.cuh, forwarded to this build's pk/config.cuh (pkt programs and tests
// that include "../include/config.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/config.cuh>
