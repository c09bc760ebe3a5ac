// pk::OpTraits<OpCode> (pkt include/op_traits.cuh:8-15): the plugin point. In
// libpkt_b200 every opcode's load / compute / store runs inside the precompiled
// sm_100a megakernel; the host-side specialisations carry the Args type so task
// lists are built exactly as with pkt (encode_args<OpTraits<Op>::Args>). A new op
// is added by giving it an opcode, an Args struct here and a case in the
// megakernel's dispatch (pkt_b200/csrc/megakernel.cu).
#pragma once

#include "task.cuh"

namespace pk {
template <OpCode Code>
struct OpTraits;
}  // namespace pk
