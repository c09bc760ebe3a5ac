// pkt's include/op_traits.cuh, forwarded to this build's pk/op_traits.cuh (pkt programs and tests
// that include "../include/op_traits.cuh" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/op_traits.cuh>
