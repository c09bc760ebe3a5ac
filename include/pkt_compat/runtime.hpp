// pkt's include/runtime.hpp, forwarded to this build's pk/runtime.hpp (pkt programs and tests
// that include "../include/runtime.hpp" compile unchanged with this directory as
// their include/).
#pragma once
#include <pk/runtime.hpp>
