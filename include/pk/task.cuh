// pk::Task, byte-identical to pkt's 96-byte descriptor (pkt include/task.cuh:11-66)
// and to pkt_task in pkt_b200.h. reserved[0..1] carry this build's optional
// second dependency token (0 keeps pkt's semantics).
#pragma once

#include <cstdint>
#include <cstring>
#include <type_traits>

#include "../pkt_b200.h"
#include "config.cuh"

namespace pk {

enum class OpCode : std::uint16_t {
  Invalid = 0,
  ZeroMemory = 1,
  Axpy = 2,
  Gemm = 3,
  LinearForward = 10,
  MSELoss = 11,
  LinearBackward = 12,
  SGDUpdate = 13,
  BiasSGD = 20,
  LossReduce = 21,
  SGDMixed = 22,
};

struct TaskHeader {
  OpCode opcode{OpCode::Invalid};
  std::uint16_t arg_bytes{0};
  std::uint32_t user_tag{0};
  std::uint16_t buffer_read_id{0};
  std::uint16_t buffer_write_id{0};
  std::uint32_t wait_count{0};
  std::uint32_t read_epoch{0};
  std::uint32_t write_epoch{0};
  std::uint32_t reserved[2]{0, 0};
};

struct alignas(16) Task {
  TaskHeader header;
  std::uint8_t args[Config::kArgBytes];
};

static_assert(sizeof(TaskHeader) == 32, "TaskHeader is 32 bytes");
static_assert(sizeof(Task) == 96 && alignof(Task) == 16, "Task is 96 bytes, 16-aligned");
static_assert(sizeof(Task) == sizeof(pkt_task), "pk::Task matches the C-ABI descriptor");

template <typename Args>
__host__ __device__ inline const Args& decode_args(const Task& t) {
  static_assert(std::is_trivially_copyable_v<Args>, "Args must be trivially copyable");
  static_assert(sizeof(Args) <= Config::kArgBytes, "Args size exceeds task payload capacity");
  return *reinterpret_cast<const Args*>(t.args);
}

template <typename Args>
inline void encode_args(Task& t, OpCode opcode, const Args& args) {
  static_assert(std::is_trivially_copyable_v<Args>, "Args must be trivially copyable");
  static_assert(sizeof(Args) <= Config::kArgBytes, "Args size exceeds task payload capacity");
  t.header = TaskHeader{};
  t.header.opcode = opcode;
  t.header.arg_bytes = static_cast<std::uint16_t>(sizeof(Args));
  std::memset(t.args, 0, Config::kArgBytes);
  std::memcpy(t.args, &args, sizeof(Args));
}

}  // namespace pk
