/*
 * Forced-include shim used only when compiling the reference's own
 * preprocessing code (extension/custom_op.cpp of IDMG-Lab/Ascend-SpMM) on the
 * CPU as a test oracle.  It is TEST INFRASTRUCTURE, never part of the product.
 *
 * The reference translation unit includes "../common/pytorch_npu_helper.hpp",
 * which needs torch_npu and the CANN ACL runtime.  The build recipe
 * (oracle/build_ref.py) predefines that header's include guard
 * (PYTORCH_NPU_HELPER_HPP_) so the header body is skipped, and force-includes
 * this file first.  The only symbol custom_op.cpp then needs from the helper
 * is the EXEC_NPU_CMD launch macro (pytorch_npu_helper.hpp:516-581); it is
 * replaced by an error, because the NPU operators cannot run here.  The CPU
 * preprocessing functions (custom_op.cpp:429-1412) are compiled unmodified.
 */
#pragma once
#include <torch/extension.h>

#define EXEC_NPU_CMD(aclnn_api, ...) \
  TORCH_CHECK(false, #aclnn_api " needs an Ascend NPU; only the CPU preprocessing is built here")
