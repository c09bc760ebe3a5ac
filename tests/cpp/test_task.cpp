// Layout and codec of pk::Task (cases of pkt's tests/test_task.cu, restated).
#include <cstddef>
#include <cstring>

#include "check.hpp"
#include "pk/ops/axpy.cuh"
#include "pk/ops/linear_bwd.cuh"
#include "pk/ops/linear_fwd.cuh"
#include "pk/ops/mse.cuh"
#include "pk/ops/sgd.cuh"
#include "pk/ops/zero.cuh"
#include "pk/task.cuh"

using namespace pk;

static bool layout() {
  CHECK(alignof(Task) == 16, "Task aligned to 16");
  CHECK(sizeof(TaskHeader) == 32, "header is 32 bytes");
  CHECK(offsetof(Task, args) == 32, "args start at 32");
  CHECK(sizeof(Task) == 96, "Task is 96 bytes");
  return true;
}

static bool opcode_values() {
  CHECK(int(OpCode::Invalid) == 0 && int(OpCode::ZeroMemory) == 1 && int(OpCode::Axpy) == 2 &&
            int(OpCode::Gemm) == 3,
        "pkt opcodes 0-3");
  CHECK(int(OpCode::LinearForward) == 10 && int(OpCode::MSELoss) == 11 &&
            int(OpCode::LinearBackward) == 12 && int(OpCode::SGDUpdate) == 13,
        "pkt opcodes 10-13");
  return true;
}

static bool encode_decode_round_trip() {
  Task t{};
  std::memset(static_cast<void*>(&t), 0xAB, sizeof(t));
  AxpyArgs a{reinterpret_cast<const float*>(0x1000), reinterpret_cast<float*>(0x2000), 2.5f, 777};
  encode_args(t, OpCode::Axpy, a);
  CHECK(t.header.opcode == OpCode::Axpy, "opcode");
  CHECK(t.header.arg_bytes == sizeof(AxpyArgs), "arg_bytes");
  CHECK(t.header.buffer_read_id == 0 && t.header.wait_count == 0 && t.header.reserved[0] == 0,
        "dependency fields cleared");
  const AxpyArgs& d = decode_args<AxpyArgs>(t);
  CHECK(d.x == a.x && d.y == a.y && d.a == 2.5f && d.n == 777, "round trip");
  for (int i = sizeof(AxpyArgs); i < Config::kArgBytes; ++i) CHECK(t.args[i] == 0, "payload tail zeroed");
  return true;
}

static bool args_sizes() {
  CHECK(sizeof(AxpyArgs) == 24 && sizeof(ZeroMemoryArgs) == 16 && sizeof(SGDUpdateArgs) == 24, "small args");
  CHECK(sizeof(LinearForwardArgs) == 56 && sizeof(LinearBackwardArgs) == 56 && sizeof(MSELossArgs) == 40,
        "linear / mse args");
  CHECK(sizeof(SGDMixedArgs) <= 64 && sizeof(BiasSGDArgs) <= 64 && sizeof(LossReduceArgs) <= 64,
        "new args fit the payload");
  return true;
}

int main() {
  Case cs[] = {{"layout", layout},
               {"opcode_values", opcode_values},
               {"encode_decode_round_trip", encode_decode_round_trip},
               {"args_sizes", args_sizes}};
  return run_cases(cs, 4);
}
