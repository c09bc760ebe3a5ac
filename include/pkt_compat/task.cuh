// pkt's include/task.cuh, forwarded to this build's pk/task.cuh (pkt programs and tests
// that include "../include/task.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/task.cuh>
