// model.cu - compiled-model runtime: weight upload and preparation, the
// liveness-planned activation arena, device-resident and host-buffer
// forwards (micro-batched, copies overlapped with compute), the batch-sliced
// multi-device forward and the per-op timed forward.
//
// Replaces the generated forward()/forward_timed() of the reference
// (examples/mnist-bench/src/generated.rs:8-294, emitted by
// cargo-psp-ml/src/codegen/render.rs:14-73,446-472), whose intermediates are
// one static buffer each (render.rs:153-180).
#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "kernels.h"
#include "runtime.h"

namespace pspml {

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int64_t in_elems_of(const pspml_op_desc& d) {
  return static_cast<int64_t>(d.in_h) * d.in_w * d.in_c;
}
int64_t out_elems_of(const pspml_op_desc& d) {
  return static_cast<int64_t>(d.out_h) * d.out_w * d.out_c;
}

bool has_weights(const pspml_op_desc& d) {
  return d.kind == PSPML_OP_CONV2D || d.kind == PSPML_OP_DEPTHWISE_CONV2D ||
         d.kind == PSPML_OP_FULLY_CONNECTED;
}

int64_t filter_bytes_of(const pspml_op_desc& d) {
  switch (d.kind) {
    case PSPML_OP_CONV2D:
      return static_cast<int64_t>(d.out_c) * d.kernel_h * d.kernel_w * d.in_c;
    case PSPML_OP_DEPTHWISE_CONV2D:
      return static_cast<int64_t>(d.kernel_h) * d.kernel_w * d.in_c;
    case PSPML_OP_FULLY_CONNECTED:
      return static_cast<int64_t>(d.out_c) * in_elems_of(d);
    default:
      return 0;
  }
}

int run_op(pspml_model* m, const ModelOp& op, int64_t mb, const int8_t* src, int8_t* dst,
           cudaStream_t s) {
  if (op.rs_weights != nullptr && (reinterpret_cast<uintptr_t>(src) & 15u) == 0 &&
      (reinterpret_cast<uintptr_t>(dst) & 31u) == 0)
    return cuda_status(launch_dense_rs(op.d, op.prep, op.rs_weights, mb, src, dst,
                                       m->ctx->dev_err, m->ctx->num_sms, s),
                       "row-streamed conv");
  return cuda_status(
      launch_op(op.d, op.prep, mb, src, dst, m->ctx->dev_err, m->ctx->num_sms, s), "op launch");
}

// Output pointer of every op for one micro-batch.
void op_pointers(pspml_model* m, const int8_t* in, int8_t* out, std::vector<int8_t*>* ptrs) {
  const int n = static_cast<int>(m->ops.size());
  ptrs->resize(n);
  // The last non-reshape op (and everything after it) writes the output.
  int last_real = n - 1;
  while (last_real > 0 && m->ops[last_real].d.kind == PSPML_OP_RESHAPE) --last_real;
  for (int i = 0; i < n; ++i) {
    const ModelOp& op = m->ops[i];
    if (i >= last_real) {
      (*ptrs)[i] = out;
    } else if (op.alias_input) {
      (*ptrs)[i] = i == 0 ? const_cast<int8_t*>(in) : (*ptrs)[i - 1];
    } else {
      (*ptrs)[i] = reinterpret_cast<int8_t*>(m->arena + op.out_off);
    }
  }
}

int forward_chunk(pspml_model* m, const int8_t* in, int8_t* out, int64_t mb, cudaStream_t s,
                  std::vector<cudaEvent_t>* events) {
  std::vector<int8_t*> ptrs;
  op_pointers(m, in, out, &ptrs);
  if (events) cudaEventRecord((*events)[0], s);
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  for (size_t i = 0; i < m->ops.size(); ++i) {
    const ModelOp& op = m->ops[i];
    const int8_t* src = i == 0 ? in : ptrs[i - 1];
    if (op.fuse == 1 && op.pool_pair && aligned(src) && aligned(ptrs[i + 1])) {
      // Conv + max pool in one kernel; the pair's time is the conv's.  A
      // conv on the row-streaming kernel pools in its epilogue (32-byte
      // stores), the others on their own conv path.
      const bool rs = op.rs_weights != nullptr &&
                      (reinterpret_cast<uintptr_t>(ptrs[i + 1]) & 31u) == 0;
      const int st = cuda_status(
          rs ? launch_dense_rs(op.d, op.prep, op.rs_weights, mb, src, ptrs[i + 1],
                               m->ctx->dev_err, m->ctx->num_sms, s, true)
             : launch_conv_pool(op.d, op.prep, mb, src, ptrs[i + 1], m->ctx->dev_err,
                                m->ctx->num_sms, s),
          "fused conv + max pool");
      if (st) return st;
      if (events) {
        cudaEventRecord((*events)[i + 1], s);
        cudaEventRecord((*events)[i + 2], s);
      }
      ++i;
      continue;
    }
    // The fused depthwise + pointwise kernels store 32-byte words.
    if (op.fuse == 1 && !op.pool_pair && aligned(src) &&
        (reinterpret_cast<uintptr_t>(ptrs[i + 1]) & 31u) == 0) {
      // Depthwise + pointwise in one kernel; the pair's time is the
      // depthwise op's, the pointwise op records none.
      const ModelOp& pw = m->ops[i + 1];
      const int st = cuda_status(launch_dwpw(op.d, op.prep, pw.d, op.wpw, *op.pair_table, mb, src,
                                             ptrs[i + 1], m->ctx->dev_err, m->ctx->num_sms, s),
                                 "fused depthwise + pointwise");
      if (st) return st;
      if (events) {
        cudaEventRecord((*events)[i + 1], s);
        cudaEventRecord((*events)[i + 2], s);
      }
      ++i;
      continue;
    }
    const int st = run_op(m, op, mb, src, ptrs[i], s);
    if (st) return st;
    if (events) cudaEventRecord((*events)[i + 1], s);
  }
  return PSPML_OK;
}

// Chunk sizes of the host-buffer pipeline.  Only the first chunk's input
// copy and the last chunk's output copy run with no compute to hide them
// under, so a long batch starts with a ramp of 1/8, 1/4 and 1/2 micro-batch
// (each chunk's compute then covers the next, twice as large, chunk's copy)
// before full micro-batches: the exposed copy shrinks eightfold.
std::vector<int64_t> pipeline_chunks(int64_t batch, int64_t micro) {
  std::vector<int64_t> sizes;
  int64_t left = batch;
  if (batch >= 2 * micro)
    for (int64_t f : {8, 4, 2}) {
      const int64_t sz = micro / f;
      if (sz >= 64) {
        sizes.push_back(sz);
        left -= sz;
      }
    }
  while (left > 0) {
    const int64_t sz = std::min(micro, left);
    sizes.push_back(sz);
    left -= sz;
  }
  return sizes;
}

int ensure_pipeline(pspml_model* m) {
  if (m->s_comp != nullptr) return PSPML_OK;
  const size_t in_b = static_cast<size_t>(m->max_micro) * m->in_elems;
  const size_t out_b = static_cast<size_t>(m->max_micro) * m->out_elems;
  int st = PSPML_OK;
  for (int k = 0; k < 2 && !st; ++k) {
    st = cuda_status(cudaMalloc(&m->stage_in[k], align_up(in_b, 256)), "cudaMalloc(stage)");
    if (!st)
      st = cuda_status(cudaMalloc(&m->stage_out[k], align_up(out_b, 256)), "cudaMalloc(stage)");
    for (cudaEvent_t* e : {&m->ev_in_ready[k], &m->ev_in_free[k], &m->ev_out_ready[k],
                           &m->ev_out_free[k]})
      if (!st) st = cuda_status(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "event");
  }
  if (!st) st = cuda_status(cudaEventCreateWithFlags(&m->ev_done, cudaEventDisableTiming), "event");
  for (cudaStream_t* s : {&m->s_h2d, &m->s_comp, &m->s_d2h})
    if (!st) st = cuda_status(cudaStreamCreateWithFlags(s, cudaStreamNonBlocking), "stream");
  return st;
}

}  // namespace

}  // namespace pspml

using namespace pspml;

extern "C" {

int pspml_model_destroy(pspml_model* m) {
  if (m == nullptr) return PSPML_OK;
  cudaSetDevice(m->ctx->device);
  if (m->s_comp) cudaStreamSynchronize(m->s_comp);
  if (m->s_h2d) cudaStreamSynchronize(m->s_h2d);
  if (m->s_d2h) cudaStreamSynchronize(m->s_d2h);
  for (int k = 0; k < 2; ++k) {
    if (m->stage_in[k]) cudaFree(m->stage_in[k]);
    if (m->stage_out[k]) cudaFree(m->stage_out[k]);
    for (cudaEvent_t e : {m->ev_in_ready[k], m->ev_in_free[k], m->ev_out_ready[k],
                          m->ev_out_free[k]})
      if (e) cudaEventDestroy(e);
  }
  if (m->ev_done) cudaEventDestroy(m->ev_done);
  for (cudaEvent_t e : m->op_events) cudaEventDestroy(e);
  for (cudaStream_t s : {m->s_h2d, m->s_comp, m->s_d2h})
    if (s) cudaStreamDestroy(s);
  if (m->arena) cudaFree(m->arena);
  if (m->weights) cudaFree(m->weights);
  if (m->pair_weights) cudaFree(m->pair_weights);
  if (m->rs_weights) cudaFree(m->rs_weights);
  delete m;
  return PSPML_OK;
}

int pspml_model_create(pspml_ctx* ctx, const pspml_op_desc* ops, int32_t n_ops,
                       const void* blob, size_t blob_bytes, int32_t max_micro_batch,
                       pspml_model** out) {
  clear_error();
  if (out == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null output pointer");
  *out = nullptr;
  if (ctx == nullptr || ops == nullptr || n_ops <= 0 || max_micro_batch <= 0)
    return set_error(PSPML_ERR_INVALID_ARG, "bad model arguments");
  if (blob == nullptr && blob_bytes > 0) return set_error(PSPML_ERR_INVALID_ARG, "null blob");
  for (int i = 0; i < n_ops; ++i) {
    int st = validate_desc(&ops[i]);
    if (st) return set_error(st, "op " + std::to_string(i) + ": " + pspml_last_error());
    if (i > 0 && in_elems_of(ops[i]) != out_elems_of(ops[i - 1]))
      return set_error(PSPML_ERR_INVALID_ARG,
                       "op " + std::to_string(i) + " input size != op " +
                           std::to_string(i - 1) + " output size");
    if (i > 0 && ops[i].zp_in != ops[i - 1].zp_out)
      return set_error(PSPML_ERR_INVALID_ARG,
                       "op " + std::to_string(i) + " zero point differs from its producer's");
    if (has_weights(ops[i])) {
      const pspml_op_desc& d = ops[i];
      const int64_t fb = filter_bytes_of(d);
      const int64_t nch = d.out_c;
      const struct {
        int64_t off, bytes;
        bool required;
        const char* name;
      } t[4] = {{d.filter_off, fb, true, "filter"},
                {d.bias_off, nch * 4, false, "bias"},
                {d.mult_off, nch * 4, true, "mult"},
                {d.shift_off, nch * 4, true, "shift"}};
      for (const auto& x : t) {
        if (x.off < 0) {
          if (x.required)
            return set_error(PSPML_ERR_INVALID_ARG,
                             "op " + std::to_string(i) + ": missing " + x.name);
          continue;
        }
        if (x.off % 16 != 0 || static_cast<uint64_t>(x.off + x.bytes) > blob_bytes)
          return set_error(PSPML_ERR_INVALID_ARG, "op " + std::to_string(i) + ": " + x.name +
                                                      " offset unaligned or outside the blob");
      }
    }
  }
  int st = cuda_status(cudaSetDevice(ctx->device), "cudaSetDevice");
  if (st) return st;

  auto* m = new pspml_model();
  m->ctx = ctx;
  m->max_micro = max_micro_batch;
  m->in_elems = in_elems_of(ops[0]);
  m->out_elems = out_elems_of(ops[n_ops - 1]);
  m->ops.resize(n_ops);

  // Prepared tables (folded biases, requantisation constants, packed
  // weights) go after the blob.
  std::vector<size_t> table_off(n_ops, 0);
  size_t wbytes = align_up(blob_bytes, 256);
  for (int i = 0; i < n_ops; ++i) {
    ModelOp& op = m->ops[i];
    op.d = ops[i];
    op.in_elems = in_elems_of(ops[i]);
    op.out_elems = out_elems_of(ops[i]);
    OpPath path = choose_path(op.d, true);
    size_t need = prepared_bytes(op.d, path);
    if (path == OpPath::kTc4d && need == 0) {  // too many border classes for the tables
      path = OpPath::kDirect;
      need = prepared_bytes(op.d, path);
    }
    op.prep.path = path;
    table_off[i] = wbytes;
    wbytes += need;
  }
  st = cuda_status(cudaMalloc(&m->weights, wbytes), "cudaMalloc(weights)");
  // The upload is ordered on the preparation stream: a plain cudaMemcpy from
  // pageable memory runs on the legacy default stream and may return before
  // its DMA lands, which the context's non-blocking stream does not wait for
  // (the table-building kernels below then read stale multipliers).
  if (!st && blob_bytes > 0)
    st = cuda_status(
        cudaMemcpyAsync(m->weights, blob, blob_bytes, cudaMemcpyHostToDevice, ctx->stream),
        "weight upload");
  for (int i = 0; i < n_ops && !st; ++i) {
    ModelOp& op = m->ops[i];
    const pspml_op_desc& d = op.d;
    const int8_t* filter = nullptr;
    const int32_t *bias = nullptr, *mult = nullptr, *shift = nullptr;
    if (has_weights(d)) {
      filter = reinterpret_cast<int8_t*>(m->weights + d.filter_off);
      bias = d.bias_off >= 0 ? reinterpret_cast<int32_t*>(m->weights + d.bias_off) : nullptr;
      mult = reinterpret_cast<int32_t*>(m->weights + d.mult_off);
      shift = reinterpret_cast<int32_t*>(m->weights + d.shift_off);
    }
    st = cuda_status(prepare_op(d, op.prep.path, filter, bias, mult, shift,
                                m->weights + table_off[i], &op.prep, ctx->stream),
                     "op preparation");
    if (has_weights(d)) {
      const auto* hb = static_cast<const uint8_t*>(blob);
      op.prep.all_fast_known =
          host_all_fast(reinterpret_cast<const int32_t*>(hb + d.mult_off),
                        reinterpret_cast<const int32_t*>(hb + d.shift_off), d.out_c);
    }
  }
  if (!st) st = cuda_status(cudaStreamSynchronize(ctx->stream), "model preparation");
  // Host copies of the requant / folded-bias tables for the tensor-core ops
  // whose tables fit a kernel parameter.
  for (int i = 0; i < n_ops && !st; ++i) {
    PreparedOp& p = m->ops[i].prep;
    const int n = m->ops[i].d.out_c;
    const bool tc = p.path == OpPath::kTc2d || p.path == OpPath::kTc4d ||
                    p.path == OpPath::kDwTc || p.path == OpPath::kSmallConv;
    if (!tc || !p.all_fast_known || n > kTabRq || (p.ncls > 1 && p.ncls * n > kTabDelta))
      continue;
    std::vector<RqChannel> rq(n);
    std::vector<int32_t> bias(static_cast<size_t>(p.ncls) * n);
    st = cuda_status(cudaMemcpy(rq.data(), p.rq, static_cast<size_t>(n) * sizeof(RqChannel),
                                cudaMemcpyDeviceToHost),
                     "table copy");
    if (!st)
      st = cuda_status(cudaMemcpy(bias.data(), p.bias_eff, bias.size() * 4,
                                  cudaMemcpyDeviceToHost),
                       "table copy");
    if (st) break;
    bool low_word_fixed = true;  // every channel's C low word is 2^30 (right shift >= 2)
    for (const RqChannel& q : rq) low_word_fixed = low_word_fixed && q.c_lo == 0x40000000u;
    if (!low_word_fixed) continue;
    auto t = std::make_unique<EpiTable>();
    std::memset(t.get(), 0, sizeof(EpiTable));
    const size_t base = static_cast<size_t>(p.base_cls) * n;
    const pspml_op_desc& d = m->ops[i].d;
    const bool floor_form = (ep_flags(d.act_min, d.act_max, d.zp_out) & kEpFloor) != 0;
    for (int c = 0; c < n; ++c) {
      if (floor_form) {
        floor_entry(rq[c].m, rq[c].c_lo, rq[c].c_hi, rq[c].sr, bias[base + c], &t->mh[c],
                    &t->bs[c]);
      } else {
        t->mh[c] = make_int2(rq[c].m, rq[c].c_hi);
        t->bs[c] = make_int2(bias[base + c], rq[c].sr);
      }
    }
    if (p.ncls > 1)
      for (int k = 0; k < p.ncls; ++k)
        for (int c = 0; c < n; ++c)
          t->dbias[k * n + c] = bias[static_cast<size_t>(k) * n + c] - bias[base + c];
    p.table = t.get();
    m->tables.push_back(std::move(t));
  }

  // Constant tables of the small-channel convs with 32 outputs and a patch
  // of at most 16 bytes (the stem): requant constants, folded bias and the
  // patch-order weight words.
  for (int i = 0; i < n_ops && !st; ++i) {
    PreparedOp& p = m->ops[i].prep;
    const pspml_op_desc& d = m->ops[i].d;
    if (p.path != OpPath::kSmallConv || !p.all_fast_known || d.out_c != 32 || d.in_c != 1 ||
        d.kernel_h != 3 || d.kernel_w != 3 || p.nw < 3)
      continue;
    std::vector<RqChannel> rq(32);
    std::vector<int32_t> bias(32);
    std::vector<uint32_t> w(static_cast<size_t>(32) * p.nw);
    st = cuda_status(cudaMemcpy(rq.data(), p.rq, 32 * sizeof(RqChannel), cudaMemcpyDeviceToHost),
                     "table copy");
    if (!st)
      st = cuda_status(cudaMemcpy(bias.data(), p.bias_eff, 32 * 4, cudaMemcpyDeviceToHost),
                       "table copy");
    if (!st)
      st = cuda_status(cudaMemcpy(w.data(), p.wpack, w.size() * 4, cudaMemcpyDeviceToHost),
                       "table copy");
    if (st) break;
    bool low_word_fixed = true;
    for (const RqChannel& q : rq) low_word_fixed = low_word_fixed && q.c_lo == 0x40000000u;
    if (!low_word_fixed) continue;
    auto t = std::make_unique<SmallConvTable>();
    std::memset(t.get(), 0, sizeof(SmallConvTable));
    const bool floor_form = (ep_flags(d.act_min, d.act_max, d.zp_out) & kEpFloor) != 0;
    for (int c = 0; c < 32; ++c) {
      if (floor_form) {
        floor_entry(rq[c].m, rq[c].c_lo, rq[c].c_hi, rq[c].sr, bias[c], &t->mh[c], &t->bs[c]);
      } else {
        t->mh[c] = make_int2(rq[c].m, rq[c].c_hi);
        t->bs[c] = make_int2(bias[c], rq[c].sr);
      }
      for (int j = 0; j < 4 && j < p.nw; ++j) t->w[c][j] = w[static_cast<size_t>(c) * p.nw + j];
    }
    p.sc_table = t.get();
    m->sc_tables.push_back(std::move(t));
  }

  // Depthwise + pointwise pairs that run as one kernel: both ops hold a
  // constant table, the shapes are instantiated, and the pointwise op reads
  // only the depthwise output (the op list is a chain).
  if (!st) {
    std::vector<int> pairs;
    size_t pair_bytes = 0;
    for (int i = 0; i + 1 < n_ops; ++i) {
      ModelOp& a = m->ops[i];
      ModelOp& b = m->ops[i + 1];
      if (a.fuse || b.fuse || a.d.kind != PSPML_OP_DEPTHWISE_CONV2D) continue;
      if (a.prep.path != OpPath::kDwTc || b.prep.path != OpPath::kTc2d) continue;
      if (a.prep.table == nullptr || b.prep.table == nullptr || !a.prep.all_fast_known ||
          !b.prep.all_fast_known)
        continue;
      if (!dwpw_pair_supported(a.d, b.d) || a.prep.ncls > 9) continue;
      auto t = std::make_unique<DwPwTable>();
      std::memset(t.get(), 0, sizeof(DwPwTable));
      const int C = a.d.in_c, N = b.d.out_c;
      for (int c = 0; c < C; ++c) {
        t->dw_mh[c] = a.prep.table->mh[c];
        t->dw_bs[c] = a.prep.table->bs[c];
      }
      for (int k = 0; k < a.prep.ncls; ++k)
        for (int c = 0; c < C; ++c) t->dw_dbias[k * C + c] = a.prep.table->dbias[k * C + c];
      for (int c = 0; c < N; ++c) {
        t->pw_mh[c] = b.prep.table->mh[c];
        t->pw_bs[c] = b.prep.table->bs[c];
      }
      a.fuse = 1;
      b.fuse = 2;
      a.pair_table = t.get();
      m->pair_tables.push_back(std::move(t));
      pairs.push_back(i);
      pair_bytes += align_up(dwpw_packed_bytes(b.d), 256);
    }
    if (!pairs.empty()) {
      st = cuda_status(cudaMalloc(&m->pair_weights, pair_bytes), "cudaMalloc(pair weights)");
      size_t off = 0;
      for (int i : pairs) {
        if (st) break;
        const ModelOp& b = m->ops[i + 1];
        m->ops[i].wpw = m->pair_weights + off;
        st = cuda_status(pack_pw_kmajor(b.prep.filter, b.d.out_c, b.d.in_c,
                                        m->pair_weights + off, ctx->stream),
                         "pack pair weights");
        off += align_up(dwpw_packed_bytes(b.d), 256);
      }
      if (!st) st = cuda_status(cudaStreamSynchronize(ctx->stream), "pack pair weights");
    }
  }

  // 3x3 convs of 32/64 channels stream their input rows (each input row
  // loaded once rather than once per filter tap); their max pool, if any,
  // then runs on its own.
  if (!st) {
    std::vector<int> rs_ops;
    for (int i = 0; i < n_ops; ++i)
      if (dense_rs_supported(m->ops[i].d, m->ops[i].prep)) rs_ops.push_back(i);
    if (!rs_ops.empty()) {
      size_t bytes = 0;
      for (int i : rs_ops) bytes += align_up(conv_rs_packed_bytes(m->ops[i].d), 256);
      st = cuda_status(cudaMalloc(&m->rs_weights, bytes), "cudaMalloc(rs weights)");
      size_t off = 0;
      for (size_t k = 0; k < rs_ops.size() && !st; ++k) {
        ModelOp& op = m->ops[rs_ops[k]];
        uint8_t* w = m->rs_weights + off;
        off += align_up(conv_rs_packed_bytes(op.d), 256);
        st = cuda_status(pack_conv_rs(op.d, op.prep.filter, w, ctx->stream), "pack conv weights");
        op.rs_weights = w;
      }
      if (!st) st = cuda_status(cudaStreamSynchronize(ctx->stream), "pack conv weights");
    }
  }

  // Conv + max pool pairs that run as one kernel (the conv's epilogue
  // pools its requantised outputs).
  for (int i = 0; i + 1 < n_ops && !st; ++i) {
    ModelOp& a = m->ops[i];
    ModelOp& b = m->ops[i + 1];
    if (a.fuse || b.fuse || !conv_pool_supported(a.d, a.prep, b.d)) continue;
    a.fuse = 1;
    a.pool_pair = true;
    b.fuse = 2;
  }

  // Arena: op i's output lives from op i until the last op reading it
  // (reshapes alias their input, extending its life).  Greedy first fit by
  // descending size over the time-overlapping buffers.
  if (!st) {
    int last_real = n_ops - 1;
    while (last_real > 0 && m->ops[last_real].d.kind == PSPML_OP_RESHAPE) --last_real;
    struct Buf {
      int op;
      int64_t bytes;
      int def, last;
      int64_t off;
    };
    std::vector<Buf> bufs;
    for (int i = 0; i < last_real; ++i) {
      ModelOp& op = m->ops[i];
      if (op.d.kind == PSPML_OP_RESHAPE) {
        op.alias_input = true;
        continue;
      }
      int last = i + 1;
      while (last < n_ops && m->ops[last].d.kind == PSPML_OP_RESHAPE) ++last;
      // A fused pair reads this buffer while it writes the output of its
      // second op, so the buffer lives until that op.
      if (last < n_ops && m->ops[last].fuse == 1) ++last;
      bufs.push_back(Buf{i, static_cast<int64_t>(align_up(
                                static_cast<size_t>(max_micro_batch) * op.out_elems, 256)),
                         i, last, 0});
    }
    std::vector<int> order(bufs.size());
    for (size_t k = 0; k < order.size(); ++k) order[k] = static_cast<int>(k);
    std::sort(order.begin(), order.end(),
              [&](int a, int b) { return bufs[a].bytes > bufs[b].bytes; });
    std::vector<int> placed;
    int64_t arena = 0;
    for (int k : order) {
      Buf& b = bufs[k];
      int64_t off = 0;
      bool moved = true;
      while (moved) {
        moved = false;
        for (int j : placed) {
          const Buf& o = bufs[j];
          const bool live_overlap = !(o.last < b.def || b.last < o.def);
          const bool mem_overlap = !(o.off + o.bytes <= off || off + b.bytes <= o.off);
          if (live_overlap && mem_overlap) {
            off = o.off + o.bytes;
            moved = true;
          }
        }
      }
      b.off = off;
      placed.push_back(k);
      arena = std::max(arena, off + b.bytes);
      m->ops[b.op].out_off = off;
    }
    m->arena_bytes = static_cast<size_t>(arena);
    if (arena > 0) st = cuda_status(cudaMalloc(&m->arena, m->arena_bytes), "cudaMalloc(arena)");
  }
  if (st) {
    pspml_model_destroy(m);
    return st;
  }
  *out = m;
  return PSPML_OK;
}

int pspml_model_info(const pspml_model* m, size_t* in_bytes_per_sample,
                     size_t* out_bytes_per_sample, size_t* arena_bytes) {
  if (m == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null model");
  if (in_bytes_per_sample) *in_bytes_per_sample = static_cast<size_t>(m->in_elems);
  if (out_bytes_per_sample) *out_bytes_per_sample = static_cast<size_t>(m->out_elems);
  if (arena_bytes) *arena_bytes = m->arena_bytes;
  return PSPML_OK;
}

int pspml_model_op_fused(const pspml_model* m, int32_t op, int32_t* fused) {
  clear_error();
  if (m == nullptr || fused == nullptr || op < 0 || op >= static_cast<int32_t>(m->ops.size()))
    return set_error(PSPML_ERR_INVALID_ARG, "bad model op query");
  *fused = m->ops[op].fuse;
  return PSPML_OK;
}

int pspml_forward_device(pspml_model* m, const int8_t* dev_in, int8_t* dev_out, int64_t batch,
                         void* stream) {
  clear_error();
  if (m == nullptr || dev_in == nullptr || dev_out == nullptr || batch < 0)
    return set_error(PSPML_ERR_INVALID_ARG, "bad forward arguments");
  std::lock_guard<std::mutex> lock(m->mu);
  if (m->fail_next > 0) {
    --m->fail_next;
    return set_error(m->fail_status, "injected failure (pspml_model_fail_next)");
  }
  cudaSetDevice(m->ctx->device);
  auto s = static_cast<cudaStream_t>(stream);
  for (int64_t b0 = 0; b0 < batch; b0 += m->max_micro) {
    const int64_t mb = std::min<int64_t>(m->max_micro, batch - b0);
    const int st = forward_chunk(m, dev_in + b0 * m->in_elems, dev_out + b0 * m->out_elems, mb,
                                 s, nullptr);
    if (st) return st;
  }
  return PSPML_OK;
}

int pspml_forward_timed(pspml_model* m, const int8_t* dev_in, int8_t* dev_out, int64_t batch,
                        float* ms_per_op, void* stream) {
  clear_error();
  if (m == nullptr || dev_in == nullptr || dev_out == nullptr || ms_per_op == nullptr ||
      batch <= 0)
    return set_error(PSPML_ERR_INVALID_ARG, "bad timed-forward arguments");
  std::lock_guard<std::mutex> lock(m->mu);
  cudaSetDevice(m->ctx->device);
  const size_t n = m->ops.size();
  const int64_t chunks = (batch + m->max_micro - 1) / m->max_micro;
  const size_t need = static_cast<size_t>(chunks) * (n + 1);
  while (m->op_events.size() < need) {
    cudaEvent_t e;
    int st = cuda_status(cudaEventCreate(&e), "cudaEventCreate");
    if (st) return st;
    m->op_events.push_back(e);
  }
  auto s = static_cast<cudaStream_t>(stream);
  // Events bracket every op of every micro-batch; nothing waits on the host
  // until the last one, so the timed work runs as in pspml_forward_device.
  for (int64_t c = 0; c < chunks; ++c) {
    const int64_t b0 = c * m->max_micro;
    const int64_t mb = std::min<int64_t>(m->max_micro, batch - b0);
    std::vector<cudaEvent_t> ev(m->op_events.begin() + c * (n + 1),
                                m->op_events.begin() + (c + 1) * (n + 1));
    const int st = forward_chunk(m, dev_in + b0 * m->in_elems, dev_out + b0 * m->out_elems, mb,
                                 s, &ev);
    if (st) return st;
  }
  int st = wait_event(m->ctx, m->op_events[need - 1]);
  if (st) return st;
  for (size_t i = 0; i < n; ++i) ms_per_op[i] = 0.f;
  for (int64_t c = 0; c < chunks; ++c)
    for (size_t i = 0; i < n; ++i) {
      float ms = 0.f;
      st = cuda_status(cudaEventElapsedTime(&ms, m->op_events[c * (n + 1) + i],
                                            m->op_events[c * (n + 1) + i + 1]),
                       "cudaEventElapsedTime");
      if (st) return st;
      ms_per_op[i] += ms;
    }
  return PSPML_OK;
}

int pspml_forward(pspml_model* m, const int8_t* host_in, int8_t* host_out, int64_t batch,
                  pspml_timing* timing) {
  clear_error();
  if (m == nullptr || host_in == nullptr || host_out == nullptr || batch < 0)
    return set_error(PSPML_ERR_INVALID_ARG, "bad forward arguments");
  const auto t0 = std::chrono::steady_clock::now();
  std::lock_guard<std::mutex> lock(m->mu);
  if (m->fail_next > 0) {
    --m->fail_next;
    return set_error(m->fail_status, "injected failure (pspml_model_fail_next)");
  }
  int st = cuda_status(cudaSetDevice(m->ctx->device), "cudaSetDevice");
  if (st) return st;
  if ((st = ensure_pipeline(m))) return st;
  const std::vector<int64_t> sizes = pipeline_chunks(batch, m->max_micro);
  const int64_t chunks = static_cast<int64_t>(sizes.size());
  // Three streams: H2D of chunk c+1 and D2H of chunk c-1 run under the
  // compute of chunk c; two staging slots per direction.
  int64_t b0 = 0;
  for (int64_t c = 0; c < chunks && !st; b0 += sizes[static_cast<size_t>(c)], ++c) {
    const int k = static_cast<int>(c & 1);
    const int64_t mb = sizes[static_cast<size_t>(c)];
    const size_t in_b = static_cast<size_t>(mb * m->in_elems);
    const size_t out_b = static_cast<size_t>(mb * m->out_elems);
    if (c >= 2) cudaStreamWaitEvent(m->s_h2d, m->ev_in_free[k], 0);
    st = cuda_status(cudaMemcpyAsync(m->stage_in[k], host_in + b0 * m->in_elems, in_b,
                                     cudaMemcpyHostToDevice, m->s_h2d),
                     "H2D copy");
    if (st) break;
    cudaEventRecord(m->ev_in_ready[k], m->s_h2d);
    cudaStreamWaitEvent(m->s_comp, m->ev_in_ready[k], 0);
    if (c >= 2) cudaStreamWaitEvent(m->s_comp, m->ev_out_free[k], 0);
    st = forward_chunk(m, reinterpret_cast<int8_t*>(m->stage_in[k]),
                       reinterpret_cast<int8_t*>(m->stage_out[k]), mb, m->s_comp, nullptr);
    if (st) break;
    cudaEventRecord(m->ev_in_free[k], m->s_comp);
    cudaEventRecord(m->ev_out_ready[k], m->s_comp);
    cudaStreamWaitEvent(m->s_d2h, m->ev_out_ready[k], 0);
    st = cuda_status(cudaMemcpyAsync(host_out + b0 * m->out_elems, m->stage_out[k], out_b,
                                     cudaMemcpyDeviceToHost, m->s_d2h),
                     "D2H copy");
    if (st) break;
    cudaEventRecord(m->ev_out_free[k], m->s_d2h);
  }
  cudaEventRecord(m->ev_done, m->s_d2h);
  const int wst = wait_event(m->ctx, m->ev_done);
  if (!st) st = wst;
  if (!st) st = cuda_status(cudaGetLastError(), "forward");
  // A kernel that gave up on a bounded wait left its output incomplete:
  // report it here rather than return results that are not.
  if (!st) st = pspml_ctx_check_device(m->ctx);
  if (timing) {
    timing->total_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    timing->h2d_bytes = static_cast<double>(batch) * m->in_elems;
    timing->d2h_bytes = static_cast<double>(batch) * m->out_elems;
    timing->micro_batches = static_cast<int32_t>(chunks);
    timing->devices = 1;
    timing->rerun_shards = 0;
  }
  return st;
}

int pspml_model_fail_next(pspml_model* m, int32_t count, int32_t status) {
  clear_error();
  if (m == nullptr || count < 0 || status <= PSPML_OK || status > PSPML_ERR_DEVICE_WAIT)
    return set_error(PSPML_ERR_INVALID_ARG, "bad failure-injection arguments");
  std::lock_guard<std::mutex> lock(m->mu);
  m->fail_next = count;
  m->fail_status = status;
  return PSPML_OK;
}

int pspml_forward_sharded(pspml_model* const* models, int32_t n_models, const int8_t* host_in,
                          int8_t* host_out, int64_t batch, pspml_timing* timing) {
  clear_error();
  if (models == nullptr || n_models <= 0 || host_in == nullptr || host_out == nullptr ||
      batch < 0)
    return set_error(PSPML_ERR_INVALID_ARG, "bad sharded-forward arguments");
  for (int i = 0; i < n_models; ++i) {
    if (models[i] == nullptr) return set_error(PSPML_ERR_INVALID_ARG, "null model");
    if (models[i]->in_elems != models[0]->in_elems ||
        models[i]->out_elems != models[0]->out_elems)
      return set_error(PSPML_ERR_INVALID_ARG, "models disagree on input/output size");
  }
  const auto t0 = std::chrono::steady_clock::now();
  const int64_t in_e = models[0]->in_elems, out_e = models[0]->out_elems;
  const int64_t per = (batch + n_models - 1) / n_models;
  std::vector<int> status(n_models, PSPML_OK);
  std::vector<std::string> msgs(n_models);
  std::vector<int64_t> begin(n_models), count(n_models);
  {
    std::vector<std::thread> threads;
    for (int i = 0; i < n_models; ++i) {
      begin[i] = std::min<int64_t>(batch, i * per);
      count[i] = std::max<int64_t>(0, std::min<int64_t>(per, batch - begin[i]));
      threads.emplace_back([&, i] {
        if (count[i] <= 0) return;
        pspml_model* m = models[i];
        status[i] = pspml_forward(m, host_in + begin[i] * in_e, host_out + begin[i] * out_e,
                                  count[i], nullptr);
        if (status[i]) msgs[i] = pspml_last_error();
      });
    }
    for (auto& t : threads) t.join();
  }
  // A device whose shard failed is dropped and its slice re-run, split over
  // the devices that succeeded.  A timed-out shard is not re-run: its
  // device may still be writing into host_out.
  std::vector<int> healthy, failed;
  for (int i = 0; i < n_models; ++i) (status[i] ? failed : healthy).push_back(i);
  int st = PSPML_OK;
  for (int i : failed)
    if (status[i] == PSPML_ERR_TIMEOUT || healthy.empty()) {
      st = set_error(status[i], "device " + std::to_string(i) + ": " + msgs[i]);
      break;
    }
  int32_t rerun = 0;
  if (!st && !failed.empty()) {
    struct Part {
      int model;
      int64_t b0, cnt;
      int status = PSPML_OK;
      std::string msg;
    };
    std::vector<Part> parts;
    for (int i : failed) {
      const int64_t h = static_cast<int64_t>(healthy.size());
      const int64_t sub = (count[i] + h - 1) / h;
      for (int64_t k = 0; k < h; ++k) {
        const int64_t b0 = begin[i] + k * sub;
        const int64_t cnt = std::min<int64_t>(sub, begin[i] + count[i] - b0);
        if (cnt > 0) parts.push_back(Part{healthy[static_cast<size_t>(k)], b0, cnt});
      }
      ++rerun;
    }
    // One host thread per healthy device runs its parts in order.
    std::vector<std::thread> threads;
    for (int hm : healthy)
      threads.emplace_back([&, hm] {
        for (Part& p : parts) {
          if (p.model != hm) continue;
          pspml_model* m = models[hm];
          p.status = pspml_forward(m, host_in + p.b0 * in_e, host_out + p.b0 * out_e, p.cnt,
                                   nullptr);
          if (p.status) p.msg = pspml_last_error();
        }
      });
    for (auto& t : threads) t.join();
    for (const Part& p : parts)
      if (p.status) {
        st = set_error(p.status, "re-run on device " + std::to_string(p.model) + ": " + p.msg);
        break;
      }
  }
  if (timing) {
    timing->total_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    timing->h2d_bytes = static_cast<double>(batch) * in_e;
    timing->d2h_bytes = static_cast<double>(batch) * out_e;
    timing->micro_batches = 0;
    timing->devices = n_models;
    timing->rerun_shards = rerun;
  }
  return st;
}

}  // extern "C"
