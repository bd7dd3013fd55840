// sym_b200 -- the checked typed program.
//
// prepareProgram validates every stage against the C1 tables and
// materializes its parameters as host scalars -- the quantize reciprocal is
// formed once, in binary32, from the declared scale -- exactly as the
// reference's typed::prepareProgram (libreloc/include/reloc/TypedExecute.h:52-100,
// libreloc/src/TypedExecute.cpp:293-403). Unlike the reference, this library
// has no CPU executor: a Program is lowered to device kernels
// (sym_b200/csrc/runtime/device_plan.cpp) and every element is converted on
// the GPU. fillAt/padsSettledBy/bytesAt keep their reference meaning.
#ifndef SYM_B200_RELOC_TYPEDEXECUTE_H
#define SYM_B200_RELOC_TYPEDEXECUTE_H

#include "reloc/Bind.h"

#include <cstdint>
#include <optional>
#include <string>
#include <variant>
#include <vector>

namespace reloc {
namespace typed {

/// Stable reason code plus detail (unsupported_stage, invalid_parameter,
/// pads_not_settled, pad_not_entered, fill_crosses_channel_stage,
/// fill_type_mismatch, mixed_fills_unsupported, fill_mismatch,
/// invalid_boundary, channel_out_of_range, channel_evaluation_failed).
struct ExecutionError {
  std::string code;
  std::string message;
};

struct StageArithmetic {
  ValueTransformKind transform = ValueTransformKind::Cast;
  NumericPolicyKind policy = NumericPolicyKind::IeeeRne;
  ElementType input{};
  ElementType output{};
  std::vector<float> scale;       // dequantize: the declared scale
  std::vector<float> invScale;    // quantize: fl32(1 / scale), formed once
  std::vector<int32_t> zeroPoint; // broadcast when size() == 1
  bool perChannel = false;
  bool channelIsDim = false; // channel == one logical result coordinate
  uint32_t channelDim = 0;
  int64_t channelLength = 1;
};

struct Program {
  TypedBoundPlan plan;
  std::vector<StageArithmetic> stages;
  std::vector<int64_t> resultStrides; // dense row-major over resultExtents
  int64_t sourceElements = 0;
  int64_t resultElements = 0;
  bool needsCoordinates = false;
};

std::variant<Program, ExecutionError> prepareProgram(const TypedBoundPlan &plan);

ElementType typeAt(const Program &program, uint32_t boundary);
uint32_t widthAt(const Program &program, uint32_t boundary);
bool padsSettledBy(const Program &program, uint32_t boundary);
std::variant<std::optional<uint64_t>, ExecutionError> fillAt(const Program &program, uint32_t boundary);
int64_t bytesAt(const Program &program, uint32_t boundary, bool resultLayout);

} // namespace typed
} // namespace reloc

#endif
