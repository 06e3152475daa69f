// runtime.h - context and model objects behind the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/pspml.h"
#include "kernels.h"

struct pspml_ctx {
  int device = 0;
  int num_sms = 148;
  int64_t timeout_ms = 0;
  unsigned* dev_err = nullptr;      // device error word written by kernels
  uint8_t* workspace = nullptr;     // per-op prepared tables (folded bias, requant)
  size_t workspace_bytes = 0;
  cudaStream_t stream = nullptr;    // internal stream for synchronous work
};

namespace pspml {

// Thread-local error message plumbing.
int set_error(int status, const std::string& msg);
int cuda_status(cudaError_t e, const char* what);
void clear_error();

// Validates an op descriptor; returns PSPML_OK or an error (message set).
int validate_desc(const pspml_op_desc* d);

// Waits for `ev` honouring the context's watchdog.
int wait_event(pspml_ctx* ctx, cudaEvent_t ev);

// One prepared op of a model.
struct ModelOp {
  pspml_op_desc d{};
  PreparedOp prep;
  int64_t out_off = 0;        // arena offset of the output (bytes per micro-batch)
  int64_t out_elems = 0;      // per sample
  int64_t in_elems = 0;
  bool alias_input = false;   // reshape: output is the input buffer
  // Fused pair: 1 on the first op (which then runs both ops in one
  // kernel), 2 on the second (skipped).  The pairs are a depthwise conv
  // with the 1x1 conv after it, and (pool_pair) a conv with the 2x2 max
  // pool after it.
  int fuse = 0;
  bool pool_pair = false;
  // A 3x3 conv of 32/64 channels run on the row-streaming kernel with these
  // packed dense weights (dense_rs_supported).
  const uint8_t* rs_weights = nullptr;
  const pspml::DwPwTable* pair_table = nullptr;
  const uint8_t* wpw = nullptr;  // packed pointwise weights of the pair
};

}  // namespace pspml

struct pspml_model {
  pspml_ctx* ctx = nullptr;
  std::vector<pspml::ModelOp> ops;
  uint8_t* weights = nullptr;        // device: blob + prepared tables
  uint8_t* arena = nullptr;          // device: intermediates for one micro-batch
  size_t arena_bytes = 0;
  int32_t max_micro = 0;
  int64_t in_elems = 0, out_elems = 0;
  // host-buffer pipeline state (lazily allocated)
  uint8_t* stage_in[2] = {nullptr, nullptr};
  uint8_t* stage_out[2] = {nullptr, nullptr};
  cudaStream_t s_h2d = nullptr, s_comp = nullptr, s_d2h = nullptr;
  cudaEvent_t ev_in_ready[2] = {}, ev_in_free[2] = {}, ev_out_ready[2] = {}, ev_out_free[2] = {};
  cudaEvent_t ev_done = nullptr;
  std::vector<cudaEvent_t> op_events;
  std::vector<std::unique_ptr<pspml::EpiTable>> tables;  // constant-table epilogues
  std::vector<std::unique_ptr<pspml::DwPwTable>> pair_tables;
  std::vector<std::unique_ptr<pspml::SmallConvTable>> sc_tables;
  uint8_t* pair_weights = nullptr;  // device: packed pointwise weights of fused pairs
  uint8_t* rs_weights = nullptr;    // device: packed dense weights of row-streamed convs
  // Host-side failure injection (pspml_model_fail_next): the next
  // `fail_next` forward calls return `fail_status` without touching the GPU.
  int32_t fail_next = 0;
  int32_t fail_status = 0;
  std::mutex mu;
};
