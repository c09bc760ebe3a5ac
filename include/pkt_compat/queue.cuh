// pkt's include/queue.cuh, forwarded to this build's pk/queue.cuh (pkt programs and tests
// that include "../include/queue.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/queue.cuh>
