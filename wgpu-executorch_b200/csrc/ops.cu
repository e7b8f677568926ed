// Operator registry: the recordIn of every reference operator this engine
// serves, keyed by ExecuTorch name (src/shaders/index.ts:39-60). Each
// recorder validates its positional args with the reference's checks and
// messages, resolves the kernel variant, and appends Commands whose
// parameters are fixed at record time (the reference writes its uniform
// buffers at record time too, src/context.ts:101-115).
#include <cstring>

#include "internal.h"
#include "umma_conv.h"

namespace wgx {

// ----------------------------------------------------------- arg helpers
static const wgx_arg &arg_at(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  if (i >= a.size()) fail(std::string(op) + ": missing argument " + std::to_string(i));
  return a[i];
}
static wgx_tensor *tensor_arg(const std::vector<wgx_arg> &a, size_t i, const char *op,
                              const char *what) {
  const wgx_arg &x = arg_at(a, i, op);
  if (x.kind != WGX_ARG_TENSOR || !x.v.tensor)
    fail(std::string(op) + ": " + what + " must be a Tensor");
  return x.v.tensor;
}
static wgx_tensor *opt_tensor_arg(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  const wgx_arg &x = arg_at(a, i, op);
  if (x.kind == WGX_ARG_NULL) return nullptr;
  if (x.kind != WGX_ARG_TENSOR) fail(std::string(op) + ": expected Tensor or undefined");
  return x.v.tensor;
}
static double number_arg(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  const wgx_arg &x = arg_at(a, i, op);
  if (x.kind == WGX_ARG_NUMBER) return x.v.number;
  if (x.kind == WGX_ARG_BOOL) return x.v.boolean ? 1.0 : 0.0;
  fail(std::string(op) + ": expected a number for argument " + std::to_string(i));
}
static bool opt_number_arg(const std::vector<wgx_arg> &a, size_t i, const char *op, double *v) {
  const wgx_arg &x = arg_at(a, i, op);
  if (x.kind == WGX_ARG_NULL) return false;
  *v = number_arg(a, i, op);
  return true;
}
static bool bool_arg(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  const wgx_arg &x = arg_at(a, i, op);
  if (x.kind == WGX_ARG_BOOL) return x.v.boolean != 0;
  if (x.kind == WGX_ARG_NUMBER) return x.v.number != 0;
  if (x.kind == WGX_ARG_NULL) return false;
  fail(std::string(op) + ": expected a boolean for argument " + std::to_string(i));
}
static std::vector<int64_t> list_arg(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  const wgx_arg &x = arg_at(a, i, op);
  if (x.kind == WGX_ARG_NULL) return {};
  if (x.kind == WGX_ARG_NUMBER) return {int64_t(x.v.number)};
  if (x.kind != WGX_ARG_INT_LIST) fail(std::string(op) + ": expected an int list");
  return std::vector<int64_t>(x.v.ints, x.v.ints + x.count);
}
static bool is_float(int dt) { return dt == WGX_FLOAT32 || dt == WGX_FLOAT16; }

// Shared per-op device allocations that outlive recording (packed weights).
static void *persistent_alloc(wgx_context *ctx, uint64_t bytes) { return ctx->alloc_device(bytes); }

// ------------------------------------------------------------- aten.mm
// src/shaders/mm/index.ts:32-93
static void record_mm(wgx_context *ctx, const std::vector<wgx_arg> &args) {
  const char *name = "aten.mm.default";
  wgx_tensor *a = tensor_arg(args, 0, name, "in1");
  wgx_tensor *b = tensor_arg(args, 1, name, "in2");
  wgx_tensor *out = tensor_arg(args, 2, name, "out");
  if (!is_float(a->dtype) || b->dtype != a->dtype || out->dtype != a->dtype)
    fail(std::string(name) + ": Tensors must have matching float32 or float16 dtype");
  if (a->ndim != 2 || b->ndim != 2 || out->ndim != 2)
    fail(std::string(name) + ": Tensors must be 2D matrices");
  int64_t m = a->shape[0], k1 = a->shape[1], k2 = b->shape[0], n = b->shape[1];
  if (k1 != k2)
    fail(std::string(name) + ": Matrix inner dimensions must match (" + std::to_string(k1) +
         " !== " + std::to_string(k2) + ")");
  if (out->shape[0] != m || out->shape[1] != n)
    fail(std::string(name) + ": Output shape [" + std::to_string(out->shape[0]) + ", " +
         std::to_string(out->shape[1]) + "] !== expected [" + std::to_string(m) + ", " +
         std::to_string(n) + "]");
  int dtype = a->dtype;
  const void *pa = a->data(), *pb = b->data();
  void *po = out->data();
  Command c;
  c.name = name;
  c.workspace_bytes = mm_scratch_bytes(m, n, k1, dtype);
  c.kernel_launches = c.workspace_bytes ? 2 : 1;
  c.run = [=](const ExecEnv &env) {
    launch_mm(pa, pb, po, m, n, k1, dtype, env.workspace, env.workspace_bytes, env.stream);
  };
  ctx->commands.push_back(std::move(c));
}

// ------------------------------------------------- convolution recorders
static void parse_hw(const std::vector<int64_t> &v, const char *name, const char *what, int *h,
                     int *w) {
  if (v.size() == 1) {
    *h = *w = int(v[0]);
  } else if (v.size() == 2) {
    *h = int(v[0]);
    *w = int(v[1]);
  } else {
    fail(std::string(name) + ": " + what + " must be 1 or 2 elements");
  }
}

// "<op>/<variant> B,IC,HxW->OC,OHxOW kKHxKW sS gG": the per-command label
// that profiling reports.
static std::string conv_label(const char *name, const wgx_conv2d_params &p, int variant) {
  static const char *variants[] = {"?", "umma", "gemm", "depthwise", "direct", "pointwise1"};
  char buf[192];
  snprintf(buf, sizeof buf, "%s/%s %d,%d,%dx%d->%d,%dx%d k%dx%d s%d g%d%s", name,
           variants[(variant >= 1 && variant <= 5) ? variant : 0], p.B, p.IC, p.IH, p.IW, p.OC,
           p.OH, p.OW, p.KH, p.KW, p.sH, p.groups, p.act == WGX_ACT_SILU ? " silu" : "");
  return buf;
}

// Append the command(s) of one forward convolution. Weights held by a
// program constant are packed once now; user weights are re-packed inside
// the graph on every submit so later setData calls are honoured (the
// reference reads the weight buffer at dispatch time).
static void append_conv(wgx_context *ctx, const char *name, const wgx_conv2d_params &p,
                        wgx_tensor *in, wgx_tensor *weight, wgx_tensor *bias, wgx_tensor *out) {
  wgx_conv2d_plan plan = plan_conv2d(p);
  const void *pin = in->data(), *pw = weight->data();
  const void *pbias = bias ? bias->data() : nullptr;
  void *pout = out->data();
  Command c;
  c.name = conv_label(name, p, plan.variant);
  if (plan.variant == WGX_CONV_UMMA) {
    uint64_t wbytes = umma_conv_packed_weight_bytes(p);
    void *packed = persistent_alloc(ctx, wbytes);
    bool constant = weight->buffer->constant;
    if (constant) {
      umma_conv_pack_weights(p, static_cast<const __half *>(pw), packed, ctx->stream);
      check_cuda(cudaStreamSynchronize(ctx->stream), "pack weights");
    }
    // program-level links (see ConvRecordLink)
    const ConvRecordLink *lk = ctx->conv_link;
    UmmaLink link{};
    bool linked = false, has_consumer = false;
    wgx_conv2d_params consumer{};
    void *in_xs = nullptr;
    if (lk) {
      if (lk->out_xs) {
        consumer = lk->consumer;
        link.consumer_xs = lk->out_xs;
        has_consumer = linked = true;
      }
      if (lk->in_xs) {
        if (!constant) fail(std::string(name) + ": linked input needs constant weights");
        in_xs = lk->in_xs;
        link.xs_ready = linked = true;
      }
      if (lk->resid) {
        link.resid = static_cast<const __half *>(lk->resid->data());
        linked = true;
      }
      if (!lk->split.empty()) {
        if (lk->split.size() > 4) fail(std::string(name) + ": too many output pieces");
        link.nout = int(lk->split.size());
        for (size_t k = 0; k < lk->split.size(); ++k) {
          link.outp[k] = static_cast<__half *>(lk->split[k]->data());
          link.out_ch[k] = int(lk->split[k]->shape[1]);
        }
        linked = true;
      }
      if (!lk->cat.empty()) {
        if (lk->cat.size() > 8) fail(std::string(name) + ": too many concatenated inputs");
        link.nsrc = int(lk->cat.size());
        for (size_t k = 0; k < lk->cat.size(); ++k) {
          link.src[k] = static_cast<const __half *>(lk->cat[k]->data());
          link.src_ch[k] = int(lk->cat[k]->shape[1]);
        }
        linked = true;
      }
    }
    // outputs written over an input: stage the input first (no direct mode)
    {
      // (an output written into a consumer's dedicated re-layout buffer
      // overlaps nothing; a split output replaces `out`)
      // A 1x1 tile reads and writes only its own positions and writes after
      // all of its loads completed, so an output over an input of the same
      // shape is safe for the direct mode; other overlaps are not.
      auto same_shape = [](const wgx_tensor *a, const wgx_tensor *b) {
        if (a->ndim != b->ndim) return false;
        for (int d = 0; d < a->ndim; ++d)
          if (a->shape[d] != b->shape[d]) return false;
        return true;
      };
      // (a linked concatenation is read from its sources, never from `in`)
      std::vector<const wgx_tensor *> in_t, out_t;
      if (lk && !lk->cat.empty())
        in_t.assign(lk->cat.begin(), lk->cat.end());
      else
        in_t.push_back(in);
      if (!(lk && (lk->out_xs || !lk->split.empty()))) out_t.push_back(out);
      if (lk)
        for (auto *t : lk->split) out_t.push_back(t);
      for (auto *o : out_t)
        for (auto *i : in_t)
          if (o->buffer == i->buffer && !same_shape(o, i)) link.allow_direct = false;
      if (!link.allow_direct) linked = true;
    }
    // program links in the label: "[xs<]" input written by its producer,
    // "[->xs]" output written into the consumer's input, "[catN]" N
    // concatenated sources, "[+res]" residual add, "[splitN]" N output pieces,
    // "[staged]" no direct mode
    if (has_consumer) c.name += " [->xs]";
    if (in_xs) c.name += " [xs<]";
    if (link.nsrc) c.name += " [cat" + std::to_string(link.nsrc) + "]";
    if (link.resid) c.name += " [+res]";
    if (link.nout) c.name += " [split" + std::to_string(link.nout) + "]";
    if (!link.allow_direct) c.name += " [staged]";
    c.workspace_bytes = in_xs ? 0 : umma_conv_input_bytes(p);
    c.kernel_launches = in_xs ? 1 : 2;
    c.run = [=](const ExecEnv &env) {
      UmmaLink l = link;
      if (has_consumer) l.consumer = &consumer;
      umma_conv_run(p, static_cast<const __half *>(pin), packed,
                    constant ? nullptr : static_cast<const __half *>(pw),
                    static_cast<const __half *>(pbias), static_cast<__half *>(pout),
                    in_xs ? in_xs : env.workspace, env.stream, linked ? &l : nullptr);
    };
  } else {
    c.kernel_launches = plan.n_launches;
    c.run = [=](const ExecEnv &env) {
      launch_conv2d(p, pin, pw, nullptr, pbias, pout, nullptr, 0, env.stream);
    };
  }
  ctx->commands.push_back(std::move(c));
}

// src/shaders/convolution/index.ts:58-310. `act` is WGX_ACT_NONE for the
// operator itself; the program fusion pass passes WGX_ACT_SILU when the
// convolution output only feeds sigmoid -> mul.
void record_convolution_act(wgx_context *ctx, const std::vector<wgx_arg> &args, int act) {
  const char *name = "aten.convolution.default";
  wgx_tensor *in = tensor_arg(args, 0, name, "input");
  wgx_tensor *weight = tensor_arg(args, 1, name, "weight");
  wgx_tensor *bias = opt_tensor_arg(args, 2, name);
  auto stride = list_arg(args, 3, name);
  auto padding = list_arg(args, 4, name);
  auto dilation = list_arg(args, 5, name);
  bool transposed = bool_arg(args, 6, name);
  auto out_pad = list_arg(args, 7, name);
  int groups = int(number_arg(args, 8, name));
  wgx_tensor *out = tensor_arg(args, 9, name, "out");

  if (!is_float(in->dtype) || weight->dtype != in->dtype || out->dtype != in->dtype)
    fail(std::string(name) + ": Tensors must have matching float32 or float16 dtype");
  if (bias && bias->dtype != in->dtype)
    fail(std::string(name) + ": bias dtype must match input dtype");
  if (in->ndim != 4 || weight->ndim != 4 || out->ndim != 4)
    fail(std::string(name) + ": expected 4D tensors for input, weight, and output");
  int sH, sW, pH, pW, dH, dW, opH, opW;
  parse_hw(stride, name, "stride", &sH, &sW);
  parse_hw(padding, name, "padding", &pH, &pW);
  parse_hw(dilation, name, "dilation", &dH, &dW);
  parse_hw(out_pad, name, "output_padding", &opH, &opW);
  if (groups < 1) fail(std::string(name) + ": groups must be >= 1");
  if (sH <= 0 || sW <= 0) fail(std::string(name) + ": stride must be positive");
  int b = int(in->shape[0]), ic = int(in->shape[1]), ih = int(in->shape[2]),
      iw = int(in->shape[3]);
  int oc, kh = int(weight->shape[2]), kw = int(weight->shape[3]);
  if (transposed) {
    int ocpg = int(weight->shape[1]);
    oc = ocpg * groups;
    if (weight->shape[0] != ic)
      fail(std::string(name) + ": weight dim0 !== IC (" + std::to_string(weight->shape[0]) +
           " != " + std::to_string(ic) + ")");
    if (opH >= sH || opW >= sW) fail(std::string(name) + ": output_padding >= stride");
    int eoh = (ih - 1) * sH - 2 * pH + dH * (kh - 1) + opH + 1;
    int eow = (iw - 1) * sW - 2 * pW + dW * (kw - 1) + opW + 1;
    if (out->shape[2] != eoh || out->shape[3] != eow)
      fail(std::string(name) + ": expected output spatial [" + std::to_string(eoh) + ", " +
           std::to_string(eow) + "]");
  } else {
    oc = int(weight->shape[0]);
    if (opH != 0 || opW != 0)
      fail(std::string(name) + ": non-zero output_padding unsupported for non-transposed conv");
    if (ic % groups != 0 || weight->shape[1] * groups != ic)
      fail(std::string(name) + ": weight in-ch (" + std::to_string(weight->shape[1]) +
           ") != IC/groups (" + std::to_string(double(ic) / groups) + ")");
    int ohn = ih + 2 * pH - dH * (kh - 1) - 1, own = iw + 2 * pW - dW * (kw - 1) - 1;
    if (ohn < 0 || own < 0)
      fail(std::string(name) + ": invalid geometry (kernel larger than input)");
    int eoh = ohn / sH + 1, eow = own / sW + 1;
    if (out->shape[2] != eoh || out->shape[3] != eow)
      fail(std::string(name) + ": expected output spatial [" + std::to_string(eoh) + ", " +
           std::to_string(eow) + "]");
  }
  if (out->shape[0] != b || out->shape[1] != oc)
    fail(std::string(name) + ": output batch/channels mismatch");
  if (bias && bias->numel < oc) fail(std::string(name) + ": bias must have OC elements");
  if (!transposed && oc % groups) fail(std::string(name) + ": OC not divisible by groups");

  wgx_conv2d_params p{};
  p.B = b;
  p.IC = ic;
  p.IH = ih;
  p.IW = iw;
  p.OC = oc;
  p.OH = int(out->shape[2]);
  p.OW = int(out->shape[3]);
  p.KH = kh;
  p.KW = kw;
  p.sH = sH;
  p.sW = sW;
  p.pH = pH;
  p.pW = pW;
  p.dH = dH;
  p.dW = dW;
  p.groups = groups;
  p.has_bias = bias != nullptr;
  p.dtype = in->dtype;
  p.act = act;
  p.out_min = -INFINITY;
  p.out_max = INFINITY;
  if (transposed) {
    if (act != WGX_ACT_NONE) fail(std::string(name) + ": fused activation on transposed conv");
    const void *pin = in->data(), *pw = weight->data();
    const void *pbias = bias ? bias->data() : nullptr;
    void *pout = out->data();
    Command c;
    c.name = name;
    c.kernel_launches = 1;
    c.run = [=](const ExecEnv &env) {
      launch_conv_transpose2d(p, opH, opW, pin, pw, pbias, pout, env.stream);
    };
    ctx->commands.push_back(std::move(c));
    return;
  }
  append_conv(ctx, name, p, in, weight, bias, out);
}

// src/shaders/conv-with-clamp/index.ts:60-319
static void record_conv_with_clamp(wgx_context *ctx, const std::vector<wgx_arg> &args) {
  const char *name = "et_vk.conv_with_clamp.default";
  wgx_tensor *in = tensor_arg(args, 0, name, "input");
  wgx_tensor *weight = tensor_arg(args, 1, name, "weight");
  wgx_tensor *bias = opt_tensor_arg(args, 2, name);
  auto stride = list_arg(args, 3, name);
  auto padding = list_arg(args, 4, name);
  auto dilation = list_arg(args, 5, name);
  bool transposed = bool_arg(args, 6, name);
  auto out_pad = list_arg(args, 7, name);
  int groups = int(number_arg(args, 8, name));
  double vmin = -INFINITY, vmax = INFINITY;
  opt_number_arg(args, 9, name, &vmin);
  opt_number_arg(args, 10, name, &vmax);
  wgx_tensor *out = tensor_arg(args, 11, name, "out");

  if (!is_float(in->dtype) || weight->dtype != in->dtype || out->dtype != in->dtype)
    fail(std::string(name) + ": Tensors must have matching float32 or float16 dtype");
  if (in->ndim != 4 || weight->ndim != 4 || out->ndim != 4)
    fail(std::string(name) + ": expected 4D tensors for input, weight, and output");
  if (bias && bias->dtype != in->dtype)
    fail(std::string(name) + ": bias dtype must match input dtype");
  if (transposed) fail(std::string(name) + ": transposed conv is unsupported in conv_with_clamp");
  if (groups < 1) fail(std::string(name) + ": groups must be >= 1");
  int sH, sW, pH, pW, dH, dW, opH, opW;
  parse_hw(stride, name, "stride", &sH, &sW);
  parse_hw(padding, name, "padding", &pH, &pW);
  parse_hw(dilation, name, "dilation", &dH, &dW);
  if (sH <= 0 || sW <= 0) fail(std::string(name) + ": stride must be positive");
  int n = int(in->shape[0]), ic = int(in->shape[1]), hin = int(in->shape[2]),
      win = int(in->shape[3]);
  int oc = int(weight->shape[0]), kh = int(weight->shape[2]), kw = int(weight->shape[3]);
  for (auto v : out_pad)
    if (v != 0)
      fail(std::string(name) + ": non-zero output_padding unsupported for non-transposed conv");
  (void)opH;
  (void)opW;
  int icpg = int(weight->shape[1]);
  if (ic % groups != 0 || oc % groups != 0 || icpg * groups != ic)
    fail(std::string(name) + ": bad shape (IC/groups mismatch)");
  int heff = hin + 2 * pH - dH * (kh - 1) - 1, weff = win + 2 * pW - dW * (kw - 1) - 1;
  if (heff < 0 || weff < 0)
    fail(std::string(name) + ": invalid geometry (kernel larger than input)");
  int eh = heff / sH + 1, ew = weff / sW + 1;
  if (out->shape[2] != eh || out->shape[3] != ew)
    fail(std::string(name) + ": output dims inconsistent with conv2d formula");
  if (bias && bias->shape[0] != oc) fail(std::string(name) + ": bias must be fp32 [OC]");
  if (out->shape[0] != n || out->shape[1] != oc)
    fail(std::string(name) + ": output batch/channels mismatch");

  wgx_conv2d_params p{};
  p.B = n;
  p.IC = ic;
  p.IH = hin;
  p.IW = win;
  p.OC = oc;
  p.OH = eh;
  p.OW = ew;
  p.KH = kh;
  p.KW = kw;
  p.sH = sH;
  p.sW = sW;
  p.pH = pH;
  p.pW = pW;
  p.dH = dH;
  p.dW = dW;
  p.groups = groups;
  p.has_bias = bias != nullptr;
  p.dtype = in->dtype;
  p.act = WGX_ACT_CLAMP;
  // the params block stores min/max as f32 words (index.ts:162-163)
  p.out_min = float(vmin);
  p.out_max = float(vmax);
  append_conv(ctx, name, p, in, weight, bias, out);
}

// Elementwise operators (add/sub/mul/sigmoid/relu/hardswish) live in
// ops_elementwise.cu; whole-program data-movement ops in ops_data.cu.
void register_elementwise_ops(std::unordered_map<std::string, OpRecorder> &reg);
void register_data_ops(std::unordered_map<std::string, OpRecorder> &reg);

const std::unordered_map<std::string, OpRecorder> &op_registry() {
  static const std::unordered_map<std::string, OpRecorder> reg = [] {
    std::unordered_map<std::string, OpRecorder> r;
    r["aten.mm.default"] = record_mm;
    r["aten.convolution.default"] = [](wgx_context *c, const std::vector<wgx_arg> &a) {
      record_convolution_act(c, a, WGX_ACT_NONE);
    };
    r["et_vk.conv_with_clamp.default"] = record_conv_with_clamp;
    register_elementwise_ops(r);
    register_data_ops(r);
    return r;
  }();
  return reg;
}

}  // namespace wgx
