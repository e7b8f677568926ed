// recordProgram: the Program JSON executor.
//
// Follows src/context.ts:219-317 step by step:
//   1. argument count check                          (context.ts:226-230)
//   2. one buffer per memoryPlan pool                 (context.ts:233-236)
//   3. a tensor view for every tensor value: constant -> dedicated, memObjId
//      -> the pool itself at offset 0, else dedicated (context.ts:239-261)
//   4. weights upload into the constants              (context.ts:264-277)
//   5. input copies user -> internal, non-Tensor inputs skipped (280-291)
//   6. the op chain through the registry + resolveArgs (292-300,
//      src/program.ts:188-224)
//   7. output copies internal -> user                 (context.ts:303-314)
//
// B200 design:
//   * pools, dedicated tensors and the weights image share ONE cudaMalloc
//     arena; every slice starts on a 256-byte boundary.
//   * constants alias their bytes inside a device copy of weights.bin that
//     is uploaded with a single pinned, asynchronous host-to-device copy.
//   * inputs that no operator writes are read from the caller's tensors and
//     outputs written into them (no copies; see the binding step).
//   * a fusion pass rewrites convolution -> sigmoid -> mul (SiLU) into one
//     convolution with a SiLU epilogue when the intermediate values have no
//     other reader.
#include <cstring>
#include <map>
#include <set>

#include "internal.h"
#include "json.h"
#include "umma_conv.h"

namespace wgx {

namespace {

struct PValue {
  enum Kind { Tensor, Scalar, List, TensorList, Null } kind = Null;
  // tensor
  std::vector<int64_t> shape;
  int dtype = 0;
  bool has_mem = false, has_weights = false;
  int64_t mem_obj = 0;
  uint64_t w_off = 0, w_len = 0;
  // scalar
  enum SKind { SNum, SBool, SStr } skind = SNum;
  double num = 0;
  bool b = false;
  std::string str;
  // list / tensorlist
  std::vector<int64_t> items;
};

struct POp {
  std::string name;
  std::vector<int64_t> args;
};

int parse_dtype(const std::string &s) {
  static const char *names[] = {"float32", "float16", "int32", "int8",
                                "uint8",   "bool",    "float64", "int64"};
  for (int i = 0; i < 8; ++i)
    if (s == names[i]) return i;
  fail("program: unknown dtype '" + s + "'");
}

const json::Value &need(const json::Value &o, const char *k) {
  const json::Value *v = o.get(k);
  if (!v) fail(std::string("program: missing field '") + k + "'");
  return *v;
}

int64_t as_int(const json::Value &v) {
  if (v.kind != json::Value::Number) fail("program: expected a number");
  return int64_t(v.num);
}

std::vector<int64_t> int_array(const json::Value &v) {
  if (v.kind != json::Value::Array) fail("program: expected an array");
  std::vector<int64_t> out;
  for (auto &e : v.arr) out.push_back(as_int(e));
  return out;
}

struct Program {
  std::vector<PValue> values;
  std::vector<POp> chain;
  std::vector<int64_t> input_ids, output_ids;
  std::vector<std::pair<int64_t, uint64_t>> pools;
};

Program parse_program(const char *text, uint64_t len) {
  json::Value root;
  try {
    root = json::parse(text, len);
  } catch (const std::runtime_error &e) {
    fail(e.what());
  }
  Program P;
  for (auto &v : need(root, "values").arr) {
    PValue pv;
    const std::string &t = need(v, "type").str;
    if (t == "tensor") {
      pv.kind = PValue::Tensor;
      pv.shape = int_array(need(v, "shape"));
      pv.dtype = parse_dtype(need(v, "dtype").str);
      if (auto *m = v.get("memObjId"); m && m->kind == json::Value::Number) {
        pv.has_mem = true;
        pv.mem_obj = as_int(*m);
      }
      auto *wo = v.get("weightsOffset");
      auto *wl = v.get("weightsLength");
      if (wo && wl && wo->kind == json::Value::Number && wl->kind == json::Value::Number) {
        pv.has_weights = true;
        pv.w_off = uint64_t(wo->num);
        pv.w_len = uint64_t(wl->num);
      }
    } else if (t == "scalar") {
      pv.kind = PValue::Scalar;
      const json::Value &val = need(v, "value");
      if (val.kind == json::Value::Bool) {
        pv.skind = PValue::SBool;
        pv.b = val.b;
      } else if (val.kind == json::Value::String) {
        pv.skind = PValue::SStr;
        pv.str = val.str;
      } else {
        pv.skind = PValue::SNum;
        pv.num = val.num;
      }
    } else if (t == "list") {
      pv.kind = PValue::List;
      pv.items = int_array(need(v, "items"));
    } else if (t == "tensorlist") {
      pv.kind = PValue::TensorList;
      pv.items = int_array(need(v, "items"));
    } else {
      pv.kind = PValue::Null;
    }
    P.values.push_back(std::move(pv));
  }
  for (auto &op : need(root, "chain").arr) {
    POp o;
    o.name = need(op, "name").str;
    o.args = int_array(need(op, "args"));
    P.chain.push_back(std::move(o));
  }
  P.input_ids = int_array(need(root, "inputIds"));
  P.output_ids = int_array(need(root, "outputIds"));
  for (auto &pl : need(need(root, "memoryPlan"), "pools").arr)
    P.pools.emplace_back(as_int(need(pl, "id")), uint64_t(as_int(need(pl, "size"))));
  return P;
}

uint64_t align256(uint64_t x) { return (x + 255) / 256 * 256; }

// Kernel parameters of the aten.convolution `c` (positional args) writing
// into value `out_id` with epilogue `act`; false when they cannot be formed.
bool conv_params(const Program &P, const POp &c, const std::map<int64_t, wgx_tensor *> &tensors,
                 int64_t out_id, int act, wgx_conv2d_params *pp) {
  if (c.args.size() != 10) return false;
  auto in = tensors.find(c.args[0]), w = tensors.find(c.args[1]), out = tensors.find(out_id);
  if (in == tensors.end() || w == tensors.end() || out == tensors.end()) return false;
  auto hw = [&](int64_t idx, int *h, int *wv) {
    const PValue &v = P.values[idx];
    if (v.kind != PValue::List || v.items.empty() || v.items.size() > 2) return false;
    *h = int(v.items[0]);
    *wv = int(v.items.size() == 2 ? v.items[1] : v.items[0]);
    return true;
  };
  wgx_conv2d_params p{};
  const wgx_tensor *x = in->second, *wt = w->second, *y = out->second;
  if (x->ndim != 4 || wt->ndim != 4 || y->ndim != 4) return false;
  p.B = int(x->shape[0]);
  p.IC = int(x->shape[1]);
  p.IH = int(x->shape[2]);
  p.IW = int(x->shape[3]);
  p.OC = int(wt->shape[0]);
  p.KH = int(wt->shape[2]);
  p.KW = int(wt->shape[3]);
  p.OH = int(y->shape[2]);
  p.OW = int(y->shape[3]);
  if (!hw(c.args[3], &p.sH, &p.sW) || !hw(c.args[4], &p.pH, &p.pW) ||
      !hw(c.args[5], &p.dH, &p.dW))
    return false;
  const PValue &g = P.values[c.args[8]];
  p.groups = g.kind == PValue::Scalar ? int(g.num) : 0;
  const PValue &tr = P.values[c.args[6]];
  if (tr.kind == PValue::Scalar && tr.b) return false;  // transposed
  p.has_bias = P.values[c.args[2]].kind == PValue::Tensor;
  p.dtype = x->dtype;
  p.act = act;
  p.out_min = -INFINITY;
  p.out_max = INFINITY;
  *pp = p;
  return true;
}

bool is_umma(const wgx_conv2d_params &p) {
  try {
    return plan_conv2d(p).variant == WGX_CONV_UMMA;
  } catch (const Error &) {
    return false;
  }
}

// True when the convolution `c` (aten.convolution positional args) may
// write over its own input (see conv2d_in_place_safe).
bool conv_in_place_safe(const Program &P, const POp &c,
                        const std::map<int64_t, wgx_tensor *> &tensors) {
  wgx_conv2d_params p{};
  return conv_params(P, c, tensors, c.args[9], WGX_ACT_SILU, &p) && conv2d_in_place_safe(p);
}

// SiLU fusion: conv(v) ; sigmoid(v)->s ; mul(v,s)->y  ==>  conv_silu -> y
// Returns, per chain index, 0 = record as is, 1 = fused conv head (record
// with SiLU into the mul's output), 2 = skip (absorbed).
std::vector<int> plan_fusion(const Program &P, const std::map<int64_t, wgx_tensor *> &tensors) {
  std::vector<int> mark(P.chain.size(), 0);
  std::map<int64_t, int> readers;
  for (auto &op : P.chain)
    for (auto a : op.args) {
      if (a < 0 || size_t(a) >= P.values.size()) continue;
      readers[a]++;
      if (P.values[a].kind == PValue::TensorList)
        for (auto t : P.values[a].items) readers[t]++;
    }
  std::set<int64_t> outputs(P.output_ids.begin(), P.output_ids.end());
  for (size_t i = 0; i + 2 < P.chain.size(); ++i) {
    const POp &c = P.chain[i], &s = P.chain[i + 1], &m = P.chain[i + 2];
    if (c.name != "aten.convolution.default" || c.args.size() != 10) continue;
    if (s.name != "aten.sigmoid.default" || s.args.size() != 2) continue;
    if (m.name != "aten.mul.Tensor" || m.args.size() != 3) continue;
    int64_t v = c.args[9], sv = s.args[1], y = m.args[2];
    if (s.args[0] != v) continue;
    if (!((m.args[0] == v && m.args[1] == sv) || (m.args[0] == sv && m.args[1] == v))) continue;
    // v read by conv(out) + sigmoid + mul, s by sigmoid(out) + mul
    if (readers[v] != 3 || readers[sv] != 2) continue;
    if (outputs.count(v) || outputs.count(sv)) continue;
    const PValue &tr = P.values[c.args[6]];
    if (tr.kind == PValue::Scalar && tr.b) continue;  // transposed
    auto tv = tensors.find(v), ty = tensors.find(y), tx = tensors.find(c.args[0]);
    if (tv == tensors.end() || ty == tensors.end() || tx == tensors.end()) continue;
    if (tv->second->numel != ty->second->numel || tv->second->dtype != ty->second->dtype)
      continue;
    // The fused conv writes y directly. When y shares the conv input's
    // buffer, only variants that read all of a region before writing it
    // may fuse (conv2d_in_place_safe).
    if (ty->second->buffer->dptr == tx->second->buffer->dptr &&
        !conv_in_place_safe(P, c, tensors))
      continue;
    mark[i] = 1;
    mark[i + 1] = 2;
    mark[i + 2] = 2;
    i += 2;
  }
  return mark;
}

// Producer/consumer links between tensor-core convolutions (after SiLU
// fusion), so intermediate activations skip their NCHW round trip:
//  * conv -> conv: when a convolution's output has no other reader, the
//    producer's epilogue writes the consumer's re-laid input (a dedicated
//    buffer, zeroed once here so its padding and unused channels stay zero)
//    and the consumer skips its re-layout kernel;
//  * cat -> conv: a channel concatenation immediately followed by its only
//    reader, a convolution, is not materialised; the consumer's re-layout
//    reads the pieces directly.
struct LinkPlan {
  std::map<size_t, ConvRecordLink> conv;  // chain index -> links of that convolution
  std::set<size_t> skip;                  // absorbed concatenations
};

LinkPlan plan_links(wgx_context *ctx, const Program &P,
                    const std::map<int64_t, wgx_tensor *> &tensors, const std::vector<int> &fusion) {
  LinkPlan L;
  std::map<int64_t, int> readers;
  std::map<int64_t, std::vector<size_t>> reader_ops;  // direct (non-list) readers
  for (size_t i = 0; i < P.chain.size(); ++i) {
    if (fusion[i] == 2) continue;
    const POp &op = P.chain[i];
    for (size_t k = 0; k + 1 < op.args.size(); ++k) {
      const int64_t a = op.args[k];
      if (a < 0 || size_t(a) >= P.values.size()) continue;
      readers[a]++;
      reader_ops[a].push_back(i);
      if (P.values[a].kind == PValue::TensorList)
        for (auto t : P.values[a].items) readers[t]++;
    }
  }
  std::set<int64_t> boundary(P.output_ids.begin(), P.output_ids.end());
  boundary.insert(P.input_ids.begin(), P.input_ids.end());
  // value -> producing chain index; fused heads own the mul's output
  std::map<int64_t, size_t> producer;
  auto out_of = [&](size_t i) -> int64_t {
    if (fusion[i] == 1) return P.chain[i + 2].args[2];
    return P.chain[i].args.empty() ? int64_t(-1) : P.chain[i].args.back();
  };
  for (size_t i = 0; i < P.chain.size(); ++i)
    if (fusion[i] != 2 && out_of(i) >= 0) producer[out_of(i)] = i;
  auto conv_of = [&](size_t i, wgx_conv2d_params *pp) {
    const POp &op = P.chain[i];
    if (op.name != "aten.convolution.default" || fusion[i] == 2) return false;
    return conv_params(P, op, tensors, out_of(i), fusion[i] == 1 ? WGX_ACT_SILU : WGX_ACT_NONE,
                       pp) &&
           is_umma(*pp);
  };
  for (size_t j = 0; j < P.chain.size(); ++j) {
    wgx_conv2d_params pc{};
    if (!conv_of(j, &pc)) continue;
    const int64_t x = P.chain[j].args[0];
    auto wt = tensors.find(P.chain[j].args[1]);
    if (wt == tensors.end() || !wt->second->buffer->constant) continue;
    if (readers[x] != 1 || boundary.count(x) || !producer.count(x)) continue;
    const size_t k = producer[x];
    wgx_conv2d_params pp{};
    if (k < j && conv_of(k, &pp) && umma_conv_link_ok(pp, pc)) {
      const uint64_t bytes = umma_conv_input_bytes(pc);
      void *buf = ctx->alloc_device(bytes);
      check_cuda(cudaMemsetAsync(buf, 0, bytes, ctx->stream), "link buffer");
      L.conv[k].out_xs = buf;
      L.conv[k].consumer = pc;
      L.conv[j].in_xs = buf;
      continue;
    }
    const POp &cat = P.chain[k];
    if (cat.name == "aten.cat.default" && k + 1 == j && cat.args.size() == 3 &&
        P.values[cat.args[0]].kind == PValue::TensorList) {
      const PValue &dimv = P.values[cat.args[1]];
      const int dim = dimv.kind == PValue::Scalar ? int(dimv.num) : -99;
      if (dim != 1 && dim != -3) continue;
      std::vector<wgx_tensor *> pieces;
      bool ok = P.values[cat.args[0]].items.size() <= 8;
      for (auto t : P.values[cat.args[0]].items) {
        auto it = tensors.find(t);
        if (it == tensors.end()) {
          ok = false;
          break;
        }
        const wgx_tensor *pt = it->second;
        ok = ok && pt->dtype == WGX_FLOAT16 && pt->ndim == 4 && pt->shape[0] == pc.B &&
             pt->shape[2] == pc.IH && pt->shape[3] == pc.IW && pt->shape[1] % 8 == 0;
        pieces.push_back(it->second);
      }
      if (!ok) continue;
      L.conv[j].cat = pieces;
      L.skip.insert(k);
    }
  }
  // * split: a channel split immediately after a convolution whose output
  //   it alone reads is done by the convolution's epilogue (each channel
  //   range written straight into its piece);
  // * residual: add(x, conv) immediately after a convolution whose output it
  //   alone reads is done by the convolution's epilogue (x added after the
  //   activation, the sum written to the add's output).
  auto last_of = [&](size_t i) { return fusion[i] == 1 ? i + 2 : i; };
  auto free_output = [&](size_t k) {
    auto it = L.conv.find(k);
    return it == L.conv.end() || (!it->second.out_xs && it->second.split.empty() &&
                                  !it->second.resid && !it->second.out_override);
  };
  auto same4 = [](const wgx_tensor *a, const wgx_tensor *b) {
    if (!a || !b || a->ndim != 4 || b->ndim != 4 || a->dtype != b->dtype) return false;
    for (int d = 0; d < 4; ++d)
      if (a->shape[d] != b->shape[d]) return false;
    return true;
  };
  for (size_t j = 0; j < P.chain.size(); ++j) {
    if (fusion[j] == 2 || L.skip.count(j)) continue;
    const POp &op = P.chain[j];
    if (op.name == "aten.split_with_sizes_copy.default" && op.args.size() == 4) {
      const int64_t x = op.args[0];
      if (!producer.count(x) || boundary.count(x)) continue;
      const size_t k = producer[x];
      wgx_conv2d_params pp{};
      if (!conv_of(k, &pp) || !free_output(k)) continue;
      const PValue &dimv = P.values[op.args[2]];
      const int dim = dimv.kind == PValue::Scalar ? int(dimv.num) : -99;
      const PValue &outs = P.values[op.args[3]];
      if ((dim != 1 && dim != -3) || outs.kind != PValue::TensorList || outs.items.empty() ||
          outs.items.size() > 4)
        continue;
      // every reader of x must be a split into the same channel ranges (the
      // exported graph may split one value twice); this one comes first
      std::vector<size_t> splits;
      bool all_split = readers[x] == int(reader_ops[x].size());
      for (size_t r : reader_ops[x]) {
        const POp &o = P.chain[r];
        const bool same =
            o.name == op.name && o.args.size() == 4 && o.args[0] == x &&
            P.values[o.args[1]].items == P.values[op.args[1]].items &&
            P.values[o.args[2]].kind == PValue::Scalar && int(P.values[o.args[2]].num) == dim &&
            P.values[o.args[3]].kind == PValue::TensorList &&
            P.values[o.args[3]].items.size() == outs.items.size();
        all_split = all_split && same;
        splits.push_back(r);
      }
      if (!all_split || splits.empty() || splits.front() != j) continue;
      // a single split right after the convolution writes the pieces where
      // the memory plan put them; otherwise the pieces get buffers of their
      // own (the planned ones may still hold live values when the
      // convolution runs), shared by the splits' equal pieces
      const bool adjacent = splits.size() == 1 && last_of(k) + 1 == j;
      bool pieces_ok = true;
      for (size_t r : splits)
        for (auto t : P.values[P.chain[r].args[3]].items)
          pieces_ok = pieces_ok && !boundary.count(t) && tensors.count(t);
      if (!pieces_ok) continue;
      std::vector<wgx_tensor *> pieces;
      int64_t csum = 0;
      bool ok = true;
      for (auto t : outs.items) {
        auto it = tensors.find(t);
        if (it == tensors.end()) {
          ok = false;
          break;
        }
        const wgx_tensor *pt = it->second;
        ok = ok && pt->ndim == 4 && pt->dtype == WGX_FLOAT16 && pt->shape[0] == pp.B &&
             pt->shape[2] == pp.OH && pt->shape[3] == pp.OW;
        csum += pt->shape[1];
        pieces.push_back(it->second);
      }
      if (!ok || csum != pp.OC) continue;
      if (!adjacent) {
        for (size_t i = 0; i < outs.items.size(); ++i) {
          const wgx_tensor *pt = pieces[i];
          auto *b = new wgx_buffer();
          b->ctx = ctx;
          b->size = (pt->byte_length() + 3) / 4 * 4;
          b->dptr = ctx->alloc_device(b->size);
          b->usage = pt->buffer->usage;
          b->device = ctx->device;
          ctx->owned.push_back(b);
          for (size_t r : splits) tensors.at(P.values[P.chain[r].args[3]].items[i])->buffer = b;
        }
      }
      L.conv[k].split = pieces;
      for (size_t r : splits) L.skip.insert(r);
    } else if (op.name == "aten.add.Tensor" && (op.args.size() == 3 || op.args.size() == 4)) {
      if (op.args.size() == 4) {
        const PValue &al = P.values[op.args[2]];
        if (!(al.kind == PValue::Null || (al.kind == PValue::Scalar && al.num == 1.0))) continue;
      }
      auto yt = tensors.find(op.args.back());
      if (yt == tensors.end()) continue;
      for (int side = 1; side >= 0; --side) {
        const int64_t m = op.args[side], r = op.args[1 - side];
        if (!producer.count(m) || readers[m] != 1 || boundary.count(m)) continue;
        const size_t k = producer[m];
        wgx_conv2d_params pp{};
        if (!conv_of(k, &pp) || last_of(k) + 1 != j || !free_output(k)) continue;
        auto mt = tensors.find(m), rt = tensors.find(r);
        if (mt == tensors.end() || rt == tensors.end()) continue;
        if (!same4(mt->second, rt->second) || !same4(mt->second, yt->second) ||
            mt->second->dtype != WGX_FLOAT16)
          continue;
        L.conv[k].resid = rt->second;
        L.conv[k].out_override = yt->second;
        L.skip.insert(j);
        break;
      }
    }
  }
  // * private outputs: a 1x1 convolution reads its input with TMA while its
  //   epilogue writes, which is safe only when no output overlays an input
  //   of another shape. The memory plan may place the output in the buffer
  //   of a concatenation source (free once the concatenation ran, which the
  //   link above absorbs) or of an input that dies at the convolution; such
  //   an output gets a buffer of its own, so that the input need not be
  //   staged through the re-layout kernel first. Every reader of the value
  //   goes through its tensor, which now points at the new buffer.
  for (size_t j = 0; j < P.chain.size(); ++j) {
    wgx_conv2d_params pc{};
    if (!conv_of(j, &pc)) continue;
    if (pc.KH != 1 || pc.KW != 1 || pc.sH != 1 || pc.sW != 1 || pc.pH != 0 || pc.pW != 0) continue;
    auto lk = L.conv.find(j);
    const ConvRecordLink *cl = lk == L.conv.end() ? nullptr : &lk->second;
    if (cl && (cl->in_xs || cl->out_xs)) continue;  // re-laid input / output into a consumer
    auto xt = tensors.find(P.chain[j].args[0]);
    auto ot = tensors.find(out_of(j));
    if (xt == tensors.end() || ot == tensors.end()) continue;
    std::vector<const wgx_tensor *> reads;
    if (cl && !cl->cat.empty())
      reads.assign(cl->cat.begin(), cl->cat.end());
    else
      reads.push_back(xt->second);
    std::vector<wgx_tensor *> outs;
    if (cl && !cl->split.empty())
      outs = cl->split;
    else
      outs.push_back(cl && cl->out_override ? cl->out_override : ot->second);
    for (wgx_tensor *o : outs) {
      bool clash = false;
      for (const wgx_tensor *r : reads) clash = clash || (o->buffer == r->buffer && !same4(o, r));
      if (!clash) continue;
      auto *b = new wgx_buffer();
      b->ctx = ctx;
      b->size = (o->byte_length() + 3) / 4 * 4;
      b->dptr = ctx->alloc_device(b->size);
      b->usage = o->buffer->usage;
      b->device = ctx->device;
      ctx->owned.push_back(b);
      o->buffer = b;
    }
  }
  if (!L.conv.empty()) check_cuda(cudaStreamSynchronize(ctx->stream), "link buffers");
  return L;
}

// View-like copies (reshape, squeeze, unsqueeze, contiguous clone, and
// et_vk.prepack, a copy of a constant) of a dense tensor move no bytes: the output value aliases the input's storage
// and the operator records nothing. The input's storage must then outlive
// the output, so an input held in a memory-plan pool (reused once the input
// dies) first gets a buffer of its own. Program inputs and outputs keep
// their operators.
std::set<size_t> plan_aliases(wgx_context *ctx, const Program &P,
                              const std::map<int64_t, wgx_tensor *> &tensors,
                              const std::set<const wgx_buffer *> &pools) {
  static const std::set<std::string> kViews = {
      "aten.view_copy.default",      "aten.clone.default",        "aten.squeeze_copy.dims",
      "aten.squeeze_copy.dim",       "aten.squeeze_copy.default", "aten.unsqueeze_copy.default",
      "aten._unsafe_view.default",   "aten.alias_copy.default",   "et_vk.prepack.default"};
  std::set<int64_t> boundary(P.output_ids.begin(), P.output_ids.end());
  boundary.insert(P.input_ids.begin(), P.input_ids.end());
  std::set<size_t> skip;
  for (size_t i = 0; i < P.chain.size(); ++i) {
    const POp &op = P.chain[i];
    if (!kViews.count(op.name) || op.args.size() < 2) continue;
    const int64_t x = op.args.front(), o = op.args.back();
    auto xt = tensors.find(x), ot = tensors.find(o);
    if (x == o || xt == tensors.end() || ot == tensors.end() || boundary.count(o)) continue;
    wgx_tensor *tx = xt->second, *to = ot->second;
    if (tx->dtype != to->dtype || tx->numel != to->numel) continue;
    if (pools.count(tx->buffer)) {
      auto *b = new wgx_buffer();
      b->ctx = ctx;
      b->size = (tx->byte_length() + 3) / 4 * 4;
      b->dptr = ctx->alloc_device(b->size);
      b->usage = tx->buffer->usage;
      b->device = ctx->device;
      ctx->owned.push_back(b);
      tx->buffer = b;
    }
    to->buffer = tx->buffer;
    skip.insert(i);
  }
  return skip;
}

// Max-pool cascades (the SPPF block): 2-3 consecutive
// max_pool2d_with_indices of one same-size geometry (K x K, K in {3, 5, 7},
// stride 1, padding (K-1)/2, dilation 1, floor mode), each reading the
// previous one's values, run as one launch (record_maxpool_cascade).
struct PoolCascades {
  std::map<size_t, std::vector<size_t>> at;  // first op -> the ops of its cascade
};

// Whether value v is named by an operator other than `producer` (directly or
// inside a tensor list) or is a program output: a value for which neither
// holds is never observed, so its producer need not write it.
bool value_used_elsewhere(const Program &P, int64_t v, size_t producer) {
  for (int64_t o : P.output_ids)
    if (o == v) return true;
  for (size_t j = 0; j < P.chain.size(); ++j) {
    if (j == producer) continue;
    for (int64_t a : P.chain[j].args) {
      if (a == v) return true;
      if (a >= 0 && size_t(a) < P.values.size() && P.values[a].kind == PValue::TensorList)
        for (int64_t t : P.values[a].items)
          if (t == v) return true;
    }
  }
  return false;
}

PoolCascades plan_pool_cascades(const Program &P) {
  PoolCascades C;
  auto items_of = [&](int64_t v) -> const std::vector<int64_t> * {
    if (v < 0 || size_t(v) >= P.values.size()) return nullptr;
    const PValue &pv = P.values[v];
    return pv.kind == PValue::List ? &pv.items : nullptr;
  };
  auto pool_k = [&](const POp &op) -> int {  // K of a qualifying pool, or 0
    if (op.name != "aten.max_pool2d_with_indices.default" || op.args.size() != 7) return 0;
    const auto *k = items_of(op.args[1]), *s = items_of(op.args[2]), *p = items_of(op.args[3]),
               *d = items_of(op.args[4]);
    if (!k || !s || !p || !d || k->empty()) return 0;
    const int64_t K = (*k)[0];
    if (K != 3 && K != 5 && K != 7) return 0;
    auto all = [](const std::vector<int64_t> *v, int64_t x) {
      for (auto e : *v)
        if (e != x) return false;
      return !v->empty() && v->size() <= 2;
    };
    if (!all(k, K) || !all(s, 1) || !all(p, (K - 1) / 2) || !all(d, 1)) return 0;
    const PValue &cm = P.values[op.args[5]];
    if (!(cm.kind == PValue::Scalar && cm.num == 0 && !cm.b)) return 0;
    const PValue &outs = P.values[op.args[6]];
    if (outs.kind != PValue::TensorList || outs.items.size() != 2) return 0;
    return int(K);
  };
  for (size_t i = 0; i < P.chain.size();) {
    const int K = pool_k(P.chain[i]);
    if (!K) {
      ++i;
      continue;
    }
    std::vector<size_t> ops{i};
    while (ops.size() < 3 && ops.back() + 1 < P.chain.size()) {
      const POp &prev = P.chain[ops.back()], &nx = P.chain[ops.back() + 1];
      if (pool_k(nx) != K || nx.args[0] != P.values[prev.args[6]].items[0]) break;
      ops.push_back(ops.back() + 1);
    }
    if (ops.size() >= 2) C.at[i] = ops;
    i = ops.back() + 1;
  }
  return C;
}

// Attention fusion: bmm(Q, K^T) -> view -> softmax(-1) -> permute(last two)
// -> squeeze/view -> bmm(V^T, .) (the PSA block of YOLO26-N) becomes one
// fused tcgen05 kernel recorded where the second bmm stood. Every
// intermediate must have exactly one reader and not be a program output, and
// no op left between the two bmm's may write into the buffers of Q or K^T
// (the fused kernel reads them later than the first bmm did).
struct AttnPlan {
  struct Site {
    int64_t q, kt, vt, ot;
    // when an op left between the two bmm's reuses the memory of Q or K^T,
    // both are copied into these buffers where the first bmm stood
    void *q_snap = nullptr, *kt_snap = nullptr;
  };
  std::map<size_t, Site> at;        // chain index of the second bmm -> operands
  std::map<size_t, size_t> snap_at; // chain index of the first bmm -> its second bmm
  std::set<size_t> skip;
};

AttnPlan plan_attention(wgx_context *ctx, const Program &P,
                        const std::map<int64_t, wgx_tensor *> &tensors,
                        const std::vector<int> &fusion, const std::set<size_t> &already_skipped) {
  AttnPlan A;
  std::map<int64_t, std::vector<size_t>> readers;
  for (size_t i = 0; i < P.chain.size(); ++i) {
    if (fusion[i] == 2 || already_skipped.count(i)) continue;
    const POp &op = P.chain[i];
    for (size_t k = 0; k + 1 < op.args.size(); ++k) {
      const int64_t a = op.args[k];
      if (a < 0 || size_t(a) >= P.values.size()) continue;
      readers[a].push_back(i);
      if (P.values[a].kind == PValue::TensorList)
        for (auto t : P.values[a].items) readers[t].push_back(i);
    }
  }
  std::set<int64_t> outputs(P.output_ids.begin(), P.output_ids.end());
  auto T = [&](int64_t v) -> const wgx_tensor * {
    auto it = tensors.find(v);
    return it == tensors.end() ? nullptr : it->second;
  };
  // the single reader of value v, or SIZE_MAX
  auto only_reader = [&](int64_t v) -> size_t {
    auto it = readers.find(v);
    if (it == readers.end() || it->second.size() != 1 || outputs.count(v)) return SIZE_MAX;
    return it->second[0];
  };
  for (size_t i = 0; i < P.chain.size(); ++i) {
    const POp &b1 = P.chain[i];
    if (b1.name != "aten.bmm.default" || b1.args.size() != 3 || fusion[i] == 2) continue;
    const wgx_tensor *q = T(b1.args[0]), *kt = T(b1.args[1]), *s = T(b1.args[2]);
    if (!q || !kt || !s || q->ndim != 3 || kt->ndim != 3 || q->dtype != WGX_FLOAT16) continue;
    const int64_t n = q->shape[0], L = q->shape[1], dq = q->shape[2];
    if (kt->shape[0] != n || kt->shape[1] != dq || kt->shape[2] != L) continue;
    std::vector<size_t> chain_ops{i};
    size_t r1 = only_reader(b1.args[2]);
    if (r1 == SIZE_MAX || P.chain[r1].name != "aten.view_copy.default") continue;
    size_t r2 = only_reader(P.chain[r1].args.back());
    if (r2 == SIZE_MAX || P.chain[r2].name != "aten._softmax.default") continue;
    {
      const wgx_tensor *x = T(P.chain[r2].args[0]);
      const PValue &d = P.values[P.chain[r2].args[1]];
      if (!x || d.kind != PValue::Scalar || (int(d.num) != -1 && int(d.num) != x->ndim - 1))
        continue;
    }
    size_t r3 = only_reader(P.chain[r2].args.back());
    if (r3 == SIZE_MAX || P.chain[r3].name != "aten.permute_copy.default") continue;
    {
      const PValue &pv = P.values[P.chain[r3].args[1]];
      const wgx_tensor *x = T(P.chain[r3].args[0]);
      if (!x || pv.kind != PValue::List || int(pv.items.size()) != x->ndim) continue;
      bool swap_last = true;
      const int nd = x->ndim;
      for (int d = 0; d < nd; ++d) {
        const int64_t want = d == nd - 1 ? nd - 2 : d == nd - 2 ? nd - 1 : d;
        const int64_t got = pv.items[d] < 0 ? pv.items[d] + nd : pv.items[d];
        swap_last = swap_last && got == want;
      }
      if (!swap_last) continue;
    }
    size_t r4 = only_reader(P.chain[r3].args.back());
    if (r4 == SIZE_MAX || (P.chain[r4].name != "aten.squeeze_copy.dims" &&
                           P.chain[r4].name != "aten.view_copy.default"))
      continue;
    const int64_t pt = P.chain[r4].args.back();
    size_t r5 = only_reader(pt);
    if (r5 == SIZE_MAX || P.chain[r5].name != "aten.bmm.default" ||
        P.chain[r5].args.size() != 3 || P.chain[r5].args[1] != pt)
      continue;
    const wgx_tensor *vt = T(P.chain[r5].args[0]), *ot = T(P.chain[r5].args[2]),
                     *ptt = T(pt);
    if (!vt || !ot || !ptt || vt->ndim != 3 || vt->dtype != WGX_FLOAT16) continue;
    const int64_t dv = vt->shape[1];
    if (vt->shape[0] != n || vt->shape[2] != L || ptt->numel != n * L * L) continue;
    if (ot->shape[0] != n || ot->shape[1] != dv || ot->shape[2] != L) continue;
    if (!attention_supported(n, L, dq, dv)) continue;
    if (!(i < r1 && r1 < r2 && r2 < r3 && r3 < r4 && r4 < r5)) continue;
    std::set<size_t> absorbed{i, r1, r2, r3, r4};
    bool safe = true;
    for (size_t k = i + 1; k < r5 && safe; ++k) {
      if (absorbed.count(k) || fusion[k] == 2 || already_skipped.count(k)) continue;
      const int64_t o = fusion[k] == 1 ? P.chain[k + 2].args[2] : P.chain[k].args.back();
      std::vector<int64_t> outs{o};
      if (P.values[o].kind == PValue::TensorList) outs = P.values[o].items;
      for (auto t : outs) {
        const wgx_tensor *w = T(t);
        if (w && (w->buffer == q->buffer || w->buffer == kt->buffer)) safe = false;
      }
    }
    AttnPlan::Site site{b1.args[0], b1.args[1], P.chain[r5].args[0], P.chain[r5].args[2]};
    if (!safe) {
      site.q_snap = ctx->alloc_device(q->byte_length());
      site.kt_snap = ctx->alloc_device(kt->byte_length());
      A.snap_at[i] = r5;
    }
    A.at[r5] = site;
    A.skip.insert(absorbed.begin(), absorbed.end());
  }
  return A;
}

}  // namespace

static void record_program_impl(wgx_context *ctx, const char *text, uint64_t len,
                                const void *weights, uint64_t wlen, const wgx_arg *args,
                                int nargs) {
  Program P = parse_program(text, len);
  size_t n_in = P.input_ids.size(), n_out = P.output_ids.size();
  if (size_t(nargs) != n_in + n_out)
    fail("program: expected " + std::to_string(n_in + n_out) + " args, got " +
         std::to_string(nargs));

  // ---- arena layout: pools, dedicated tensors, weights image
  std::map<int64_t, uint64_t> pool_off, pool_size;
  uint64_t off = 0;
  for (auto &pl : P.pools) {
    uint64_t sz = pl.second < 4 ? 4 : (pl.second + 3) / 4 * 4;
    pool_off[pl.first] = off;
    pool_size[pl.first] = sz;
    off = align256(off + sz);
  }
  std::map<size_t, uint64_t> dedicated_off;
  for (size_t i = 0; i < P.values.size(); ++i) {
    const PValue &v = P.values[i];
    if (v.kind != PValue::Tensor) continue;
    if (v.has_weights) continue;
    if (v.has_mem) {
      if (!pool_off.count(v.mem_obj))
        fail("program: no memory pool " + std::to_string(v.mem_obj) + " for value " +
             std::to_string(i));
      continue;
    }
    int64_t numel = 1;
    for (auto d : v.shape) numel *= d;
    uint64_t sz = uint64_t(numel) * dtype_size(v.dtype);
    sz = sz < 4 ? 4 : (sz + 3) / 4 * 4;
    dedicated_off[i] = off;
    off = align256(off + sz);
  }
  uint64_t weights_off = off;
  bool any_const = false;
  for (auto &v : P.values)
    if (v.kind == PValue::Tensor && v.has_weights) {
      any_const = true;
      if (v.w_off + v.w_len > wlen)
        fail("program: constant [" + std::to_string(v.w_off) + ", +" + std::to_string(v.w_len) +
             ") lies outside weights.bin (" + std::to_string(wlen) + " bytes)");
    }
  uint64_t total = weights_off + (any_const ? align256(wlen + 4) : 0);
  char *arena = static_cast<char *>(ctx->alloc_device(total));

  const uint32_t usage = WGX_USAGE_STORAGE | WGX_USAGE_COPY_SRC | WGX_USAGE_COPY_DST;
  auto slice = [&](uint64_t o, uint64_t sz, bool constant) {
    auto *b = new wgx_buffer();
    b->ctx = ctx;
    b->dptr = arena + o;
    b->size = sz;
    b->usage = usage;
    b->device = ctx->device;
    b->owns_alloc = false;
    b->constant = constant;
    ctx->owned.push_back(b);
    return b;
  };
  std::map<int64_t, wgx_buffer *> pool_buf;
  for (auto &pl : P.pools) pool_buf[pl.first] = slice(pool_off[pl.first], pool_size[pl.first], false);

  // ---- weights: one pinned staging copy, one async H2D
  if (any_const && wlen) {
    void *pinned = nullptr;
    check_cuda(cudaHostAlloc(&pinned, wlen, cudaHostAllocDefault), "cudaHostAlloc(weights)");
    std::memcpy(pinned, weights, wlen);
    cudaError_t e = cudaMemcpyAsync(arena + weights_off, pinned, wlen, cudaMemcpyHostToDevice,
                                    ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFreeHost(pinned);
    check_cuda(e, "weights upload");
  }

  // ---- tensor views
  std::map<int64_t, wgx_tensor *> tensors;
  for (size_t i = 0; i < P.values.size(); ++i) {
    const PValue &v = P.values[i];
    if (v.kind != PValue::Tensor) continue;
    wgx_buffer *buf;
    if (v.has_weights) {
      uint64_t sz = v.w_len < 4 ? 4 : (v.w_len + 3) / 4 * 4;
      buf = slice(weights_off + v.w_off, sz, true);
    } else if (v.has_mem) {
      buf = pool_buf[v.mem_obj];
    } else {
      int64_t numel = 1;
      for (auto d : v.shape) numel *= d;
      uint64_t sz = uint64_t(numel) * dtype_size(v.dtype);
      buf = slice(dedicated_off[i], sz < 4 ? 4 : (sz + 3) / 4 * 4, false);
    }
    wgx_tensor *t = nullptr;
    if (wgx_tensor_create(ctx, v.dtype, v.shape.data(), int(v.shape.size()), buf, &t) != WGX_OK)
      fail(std::string("program: value ") + std::to_string(i) + ": " + wgx_last_error());
    ctx->program_tensors.emplace_back(t);
    tensors[int64_t(i)] = t;
  }

  // ---- zero-copy binding (B200 design): an input value that no operator
  // writes reads the caller's tensor directly, and an output value is
  // written straight into the caller's tensor, instead of the copies of
  // steps 5 and 7 (same bytes at every submit: the copies would run at
  // submit time too). Only the bound value's tensor moves: the other values
  // of its pool keep the pool. Written values are taken conservatively as
  // the last two arguments of every operator (and the items of tensor lists
  // there); a caller tensor that is both an input and an output, or whose
  // dtype or shape differs from the value's, keeps the copy.
  std::set<int64_t> written;
  for (const POp &op : P.chain) {
    const size_t na = op.args.size();
    for (size_t k = na >= 2 ? na - 2 : 0; k < na; ++k) {
      const int64_t v = op.args[k];
      if (v < 0 || size_t(v) >= P.values.size()) continue;
      written.insert(v);
      if (P.values[v].kind == PValue::TensorList)
        for (auto t : P.values[v].items) written.insert(t);
    }
  }
  std::set<const wgx_buffer *> in_bufs, out_bufs;
  for (size_t i = 0; i < n_in; ++i)
    if (args[i].kind == WGX_ARG_TENSOR) in_bufs.insert(args[i].v.tensor->buffer);
  for (size_t i = 0; i < n_out; ++i)
    if (args[n_in + i].kind == WGX_ARG_TENSOR) out_bufs.insert(args[n_in + i].v.tensor->buffer);
  auto same_layout = [](const wgx_tensor *a, const wgx_tensor *b) {
    if (a->dtype != b->dtype || a->ndim != b->ndim) return false;
    for (int d = 0; d < a->ndim; ++d)
      if (a->shape[d] != b->shape[d]) return false;
    return true;
  };
  const std::set<int64_t> prog_inputs(P.input_ids.begin(), P.input_ids.end());
  std::set<int64_t> bound_out;
  for (size_t i = 0; i < n_out; ++i) {
    const wgx_arg &dst = args[n_in + i];
    auto it = tensors.find(P.output_ids[i]);
    if (dst.kind != WGX_ARG_TENSOR || it == tensors.end()) continue;
    const int64_t v = P.output_ids[i];
    if (prog_inputs.count(v) || bound_out.count(v) || in_bufs.count(dst.v.tensor->buffer) ||
        !same_layout(it->second, dst.v.tensor))
      continue;
    bool dup = false;  // one caller tensor for two outputs: keep the copies
    for (size_t k = 0; k < n_out; ++k)
      dup = dup || (k != i && args[n_in + k].kind == WGX_ARG_TENSOR &&
                    args[n_in + k].v.tensor->buffer == dst.v.tensor->buffer);
    if (dup) continue;
    it->second->buffer = dst.v.tensor->buffer;
    bound_out.insert(v);
  }

  // ---- views alias their inputs (before the input copies: an aliased input
  // value may move to a buffer of its own)
  std::set<const wgx_buffer *> pool_set;
  for (auto &kv : pool_buf) pool_set.insert(kv.second);
  const std::set<size_t> alias_skip = plan_aliases(ctx, P, tensors, pool_set);

  // ---- input copies
  for (size_t i = 0; i < n_in; ++i) {
    if (args[i].kind != WGX_ARG_TENSOR) continue;  // non-Tensor inputs are skipped
    auto it = tensors.find(P.input_ids[i]);
    if (it == tensors.end())
      fail("program: no tensor for input value " + std::to_string(P.input_ids[i]));
    const int64_t v = P.input_ids[i];
    if (!written.count(v) && !out_bufs.count(args[i].v.tensor->buffer) &&
        same_layout(it->second, args[i].v.tensor)) {
      it->second->buffer = args[i].v.tensor->buffer;
      continue;
    }
    if (wgx_copy(ctx, args[i].v.tensor, it->second) != WGX_OK) fail(wgx_last_error());
  }

  // ---- chain
  const auto &reg = op_registry();
  std::vector<int> fusion = plan_fusion(P, tensors);
  const LinkPlan links = plan_links(ctx, P, tensors, fusion);
  const AttnPlan attn = plan_attention(ctx, P, tensors, fusion, links.skip);
  const PoolCascades pools = plan_pool_cascades(P);
  std::set<size_t> pool_skip;
  for (size_t oi = 0; oi < P.chain.size(); ++oi) {
    if (auto sn = attn.snap_at.find(oi); sn != attn.snap_at.end()) {
      // snapshot Q and K^T where the first bmm read them
      const AttnPlan::Site &site = attn.at.at(sn->second);
      const wgx_tensor *q = tensors[site.q], *kt = tensors[site.kt];
      const void *sq = q->data(), *sk = kt->data();
      void *dq_ = site.q_snap, *dk = site.kt_snap;
      const uint64_t nq = q->byte_length(), nk = kt->byte_length();
      Command c;
      c.name = "attention operand snapshot";
      c.run = [=](const ExecEnv &env) {
        check_cuda(cudaMemcpyAsync(dq_, sq, nq, cudaMemcpyDeviceToDevice, env.stream), "snapshot");
        check_cuda(cudaMemcpyAsync(dk, sk, nk, cudaMemcpyDeviceToDevice, env.stream), "snapshot");
      };
      ctx->commands.push_back(std::move(c));
      continue;
    }
    if (fusion[oi] == 2 || links.skip.count(oi) || attn.skip.count(oi) || alias_skip.count(oi) ||
        pool_skip.count(oi))
      continue;
    if (auto pc = pools.at.find(oi); pc != pools.at.end()) {
      std::vector<std::pair<wgx_tensor *, wgx_tensor *>> outs;
      bool ok = true;
      for (size_t k : pc->second) {
        const auto &items = P.values[P.chain[k].args[6]].items;
        auto v = tensors.find(items[0]), ix = tensors.find(items[1]);
        if (v == tensors.end() || ix == tensors.end()) {
          ok = false;
          break;
        }
        // indices no operator reads (the SPPF block keeps only the values)
        // are not written
        outs.emplace_back(v->second,
                          value_used_elsewhere(P, items[1], k) ? ix->second : nullptr);
      }
      auto in = tensors.find(P.chain[oi].args[0]);
      const int K = int(P.values[P.chain[oi].args[1]].items[0]);
      if (ok && in != tensors.end() && record_maxpool_cascade(ctx, in->second, outs, K)) {
        pool_skip.insert(pc->second.begin() + 1, pc->second.end());
        continue;
      }
    }
    if (auto at = attn.at.find(oi); at != attn.at.end()) {
      const wgx_tensor *q = tensors[at->second.q], *kt = tensors[at->second.kt],
                       *vt = tensors[at->second.vt], *ot = tensors[at->second.ot];
      const int64_t n = q->shape[0], L = q->shape[1], dq = q->shape[2], dv = vt->shape[1];
      const __half *pq = static_cast<const __half *>(at->second.q_snap ? at->second.q_snap
                                                                       : q->data()),
                   *pk = static_cast<const __half *>(at->second.kt_snap ? at->second.kt_snap
                                                                        : kt->data()),
                   *pv = static_cast<const __half *>(vt->data());
      __half *po = static_cast<__half *>(ot->data());
      Command c;
      c.name = "attention (bmm -> softmax -> bmm)";
      c.kernel_launches = 1;
      c.run = [=](const ExecEnv &env) { launch_attention(pq, pk, pv, po, n, L, dq, dv, env.stream); };
      ctx->commands.push_back(std::move(c));
      continue;
    }
    const POp &op = P.chain[oi];
    auto rit = reg.find(op.name);
    if (rit == reg.end()) fail("program: unknown operator '" + op.name + "'");
    // resolveArgs (src/program.ts:188-224)
    std::vector<wgx_arg> a(op.args.size());
    std::vector<std::vector<int64_t>> lists(op.args.size());
    std::vector<std::vector<wgx_tensor *>> tlists(op.args.size());
    for (size_t k = 0; k < op.args.size(); ++k) {
      int64_t idx = op.args[k];
      if (idx < 0 || size_t(idx) >= P.values.size())
        fail("program: value index " + std::to_string(idx) + " out of range in '" + op.name + "'");
      const PValue &v = P.values[idx];
      wgx_arg &x = a[k];
      std::memset(&x, 0, sizeof(x));
      switch (v.kind) {
        case PValue::Tensor: {
          auto it = tensors.find(idx);
          if (it == tensors.end())
            fail("program: no tensor for value " + std::to_string(idx) + " referenced by '" +
                 op.name + "'");
          x.kind = WGX_ARG_TENSOR;
          x.v.tensor = it->second;
          break;
        }
        case PValue::Scalar:
          if (v.skind == PValue::SBool) {
            x.kind = WGX_ARG_BOOL;
            x.v.boolean = v.b;
          } else if (v.skind == PValue::SStr) {
            x.kind = WGX_ARG_STRING;
            x.v.string = v.str.c_str();
          } else {
            x.kind = WGX_ARG_NUMBER;
            x.v.number = v.num;
          }
          break;
        case PValue::List:
          lists[k] = v.items;
          x.kind = WGX_ARG_INT_LIST;
          x.count = int32_t(lists[k].size());
          x.v.ints = lists[k].data();
          break;
        case PValue::TensorList:
          for (auto t : v.items) {
            if (t < 0 || size_t(t) >= P.values.size() || P.values[t].kind != PValue::Tensor)
              fail("program: tensorlist item " + std::to_string(t) + " is not a tensor (" +
                   op.name + ")");
            auto it = tensors.find(t);
            if (it == tensors.end())
              fail("program: no tensor for value " + std::to_string(t) + " referenced by '" +
                   op.name + "'");
            tlists[k].push_back(it->second);
          }
          x.kind = WGX_ARG_TENSOR_LIST;
          x.count = int32_t(tlists[k].size());
          x.v.tensors = tlists[k].data();
          break;
        case PValue::Null:
          x.kind = WGX_ARG_NULL;
          break;
      }
    }
    size_t before = ctx->commands.size();
    auto lk = links.conv.find(oi);
    ctx->conv_link = lk == links.conv.end() ? nullptr : &lk->second;
    try {
      if (fusion[oi] == 1) {
        // fused conv + SiLU writes straight into the mul's output
        a[9].v.tensor = tensors[P.chain[oi + 2].args[2]];
        if (ctx->conv_link && ctx->conv_link->out_override)
          a[9].v.tensor = ctx->conv_link->out_override;
        record_convolution_act(ctx, a, WGX_ACT_SILU);
      } else {
        if (ctx->conv_link && ctx->conv_link->out_override && a.size() == 10)
          a[9].v.tensor = ctx->conv_link->out_override;
        rit->second(ctx, a);
      }
    } catch (...) {
      ctx->conv_link = nullptr;
      ctx->commands.resize(before);
      throw;
    }
    ctx->conv_link = nullptr;
  }

  // ---- output copies
  for (size_t i = 0; i < n_out; ++i) {
    const wgx_arg &dst = args[n_in + i];
    auto it = tensors.find(P.output_ids[i]);
    if (dst.kind != WGX_ARG_TENSOR) fail("program: output " + std::to_string(i) + " must be a Tensor");
    if (it == tensors.end())
      fail("program: no tensor for output value " + std::to_string(P.output_ids[i]));
    if (bound_out.count(P.output_ids[i])) continue;  // written in place
    if (wgx_copy(ctx, it->second, dst.v.tensor) != WGX_OK) fail(wgx_last_error());
  }
}

}  // namespace wgx

extern "C" int wgx_record_program(wgx_context *ctx, const char *json, uint64_t json_len,
                                  const void *weights, uint64_t weights_len, const wgx_arg *args,
                                  int nargs) {
  using namespace wgx;
  try {
    clear_error();
    if (!ctx) fail("null context");
    if (ctx->destroyed) fail("WgpuExecutionContext is destroyed", WGX_ERR_DESTROYED);
    check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
    size_t before = ctx->commands.size();
    try {
      record_program_impl(ctx, json, json_len, weights, weights_len, args, nargs);
    } catch (...) {
      ctx->commands.resize(before);
      ctx->invalidate_graph();
      throw;
    }
    ctx->invalidate_graph();
    return WGX_OK;
  } catch (const Error &e) {
    return set_error(e.code, e.msg);
  } catch (const std::exception &e) {
    return set_error(WGX_ERR_INVALID, e.what());
  }
}
