// Networks: model load (named parameters -> packed GPU layers) and execution of the
// synthesis / analysis topologies of src/model/{synthesis,attention,analysis}.rs on batches of
// same-shape tiles (NHWC f16 activations in the context arena).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "api_common.h"
#include "kernels_attn.h"
#include "net.h"

namespace zjai {

namespace {

int cdiv(int a, int b) { return (a + b - 1) / b; }

}  // namespace

// ---------------------------------------------------------------------------------------------
// Loading (src/model/load.rs:11-85: names and shapes are validated like the crate's loaders)
// ---------------------------------------------------------------------------------------------

struct Loader {
  Net* net;
  std::map<std::string, const zjai_param*> byname;

  int get(const std::string& name, std::vector<int64_t> shape, const float** out) {
    auto it = byname.find(name);
    if (it == byname.end()) return fail(ZJAI_MODEL, name + ": missing");
    const zjai_param* p = it->second;
    bool ok = p->ndim == (int)shape.size();
    for (size_t i = 0; ok && i < shape.size(); ++i) ok = p->shape[i] == shape[i];
    if (!ok) {
      std::string got = "[", want = "[";
      for (int i = 0; i < p->ndim; ++i) got += std::to_string(p->shape[i]) + (i + 1 < p->ndim ? ", " : "");
      for (size_t i = 0; i < shape.size(); ++i)
        want += std::to_string(shape[i]) + (i + 1 < shape.size() ? ", " : "");
      return fail(ZJAI_MODEL, name + ": shape " + got + "], expected " + want + "]");
    }
    if (!p->data) return fail(ZJAI_MODEL, name + ": null data");
    *out = p->data;
    return ZJAI_OK;
  }

  bool has(const std::string& name) const { return byname.count(name) != 0; }

  // load::conv (load.rs:11-40) + ConvLayer::new; `ps` folds a following pixel shuffle.
  int conv(const std::string& prefix, int cin, int cout, int kh, int kw, int stride, int pad,
           int groups, bool bias, const int* extra = nullptr, int ps = 1) {
    const float *w, *b = nullptr;
    ZJAI_TRY(get(prefix + ".weight", {cout, cin / groups, kh, kw}, &w));
    if (bias) ZJAI_TRY(get(prefix + ".bias", {cout}, &b));
    else if (has(prefix + ".bias"))
      return fail(ZJAI_MODEL, prefix + ": unexpected bias in checkpoint");
    ConvLayer L;
    ZJAI_TRY(pack_conv(net->ctx, &L, w, b, cin, cout, kh, kw, stride, pad, pad, groups, extra, ps));
    net->convs[prefix] = L;
    return ZJAI_OK;
  }
  // load::conv_transpose (load.rs:64-85), stride 2, always with bias
  int convt(const std::string& prefix, int cin, int cout, int k, int pad, int out_pad,
            int post_ps = 1) {
    const float *w, *b;
    ZJAI_TRY(get(prefix + ".weight", {cin, cout, k, k}, &w));
    ZJAI_TRY(get(prefix + ".bias", {cout}, &b));
    ConvLayer L;
    ZJAI_TRY(pack_convT(net->ctx, &L, w, b, cin, cout, k, pad, out_pad, post_ps));
    net->convs[prefix] = L;
    return ZJAI_OK;
  }
  // The luma analysis's first layer (weight [cout][1][3][3], bias) as a 1x1 conv over its nine
  // taps (launch_normalize_im2col): weight [cout][9][1][1], row co holding w[co][0][ky][kx] at
  // 3 ky + kx. Packed with the same power-of-two scale rule over the same values, so its f16
  // weights and its bias are the 3x3 layer's.
  int conv_im2col(const std::string& prefix, int cout) {
    const float *w, *b;
    ZJAI_TRY(get(prefix + ".weight", {cout, 1, 3, 3}, &w));
    ZJAI_TRY(get(prefix + ".bias", {cout}, &b));
    ConvLayer L;
    ZJAI_TRY(pack_conv(net->ctx, &L, w, b, 9, cout, 1, 1, 1, 0, 0, 1, nullptr, 1));
    net->convs[prefix + "#im2col"] = L;
    return ZJAI_OK;
  }
  int vec(const std::string& name, std::vector<int64_t> shape) {
    const float* p;
    ZJAI_TRY(get(name, shape, &p));
    size_t n = 1;
    for (auto s : shape) n *= (size_t)s;
    float* d = nullptr;
    ZJAI_TRY(cuda_check(cudaMalloc(&d, n * sizeof(float)), "cudaMalloc param"));
    ZJAI_TRY(cuda_check(cudaMemcpy(d, p, n * sizeof(float), cudaMemcpyHostToDevice), "param H2D"));
    net->vecs[name] = d;
    return ZJAI_OK;
  }
  // depthwise 3x3 without bias: weights [c][1][3][3] kept as [c][9] f32
  int dw(const std::string& prefix, int c) {
    ZJAI_TRY(vec(prefix + ".weight", {c, 1, 3, 3}));
    net->vecs[prefix] = net->vecs[prefix + ".weight"];
    net->vecs.erase(prefix + ".weight");
    return ZJAI_OK;
  }

  // ResAu::load (synthesis.rs:32-57): the group count comes from the weight shape
  int resau(const std::string& prefix, int c) {
    auto it = byname.find(prefix + ".conv.weight");
    if (it == byname.end() || it->second->ndim != 4 || it->second->shape[1] <= 0 ||
        c % it->second->shape[1])
      return fail(ZJAI_MODEL, prefix + ".conv.weight: missing or malformed");
    const int groups = c / (int)it->second->shape[1];
    ZJAI_TRY(conv(prefix + ".conv", c, c, 3, 3, 1, 1, groups, false));
    return conv(prefix + ".conv2", c, c, 1, 1, 1, 0, 1, false);
  }
  int rb(const std::string& prefix, int c) {  // ResidualBlock::load (attention.rs:22-34)
    ZJAI_TRY(conv(prefix + ".conv1", c, c, 3, 3, 1, 1, 1, true));
    return conv(prefix + ".conv2", c, c, 3, 3, 1, 1, 1, true);
  }
  int cab(const std::string& prefix, int c) {  // Cab::load (attention.rs:111-120)
    ZJAI_TRY(rb(prefix + ".residual_trunk.0", c));
    ZJAI_TRY(rb(prefix + ".residual_trunk.1", c));
    ZJAI_TRY(conv(prefix + ".subscale", c, c, 3, 3, 2, 1, 1, true));
    ZJAI_TRY(rb(prefix + ".residual_mask2.0", c));
    ZJAI_TRY(rb(prefix + ".residual_mask3.0", c));
    return convt(prefix + ".upscale", c, c, 3, 1, 1);
  }
  int tb(const std::string& p, int dim) {  // TransformerBlock::load (attention.rs:294-326)
    const int hidden = 4 * dim;
    ZJAI_TRY(vec(p + ".prep_data.norm1.weight", {dim}));
    ZJAI_TRY(vec(p + ".prep_data.norm1.bias", {dim}));
    ZJAI_TRY(conv(p + ".prep_data.conv1", dim, 3 * dim, 1, 1, 1, 0, 1, false));
    ZJAI_TRY(dw(p + ".prep_data.conv2", 3 * dim));
    ZJAI_TRY(vec(p + ".attn.temperature", {4, 1, 1}));
    ZJAI_TRY(conv(p + ".attn.project_out", dim, dim, 1, 1, 1, 0, 1, false));
    // f32 copy of W_o for the per-picture fold W_o . blockdiag(A). Its f16 scale: every column
    // of A sums to at most c = dim / 4 (rows are softmax distributions), so
    // |W'| <= c max|W_o| and the packed scale of W_o divided by 2^ceil(log2 c) cannot overflow.
    const float* wo;
    ZJAI_TRY(get(p + ".attn.project_out.weight", {dim, dim, 1, 1}, &wo));
    ZJAI_TRY(vec(p + ".attn.project_out.weight", {dim, dim, 1, 1}));
    int lc = 0;
    while ((1 << lc) < dim / 4) ++lc;
    net->fold_scale[p] = std::ldexp(pow2_weight_scale(wo, (size_t)dim * dim), -lc);
    ZJAI_TRY(vec(p + ".ffn.norm1.weight", {dim}));
    ZJAI_TRY(vec(p + ".ffn.norm1.bias", {dim}));
    ZJAI_TRY(conv(p + ".ffn.project_in", dim, 2 * hidden, 1, 1, 1, 0, 1, false));
    ZJAI_TRY(dw(p + ".ffn.dwconv", 2 * hidden));
    ZJAI_TRY(conv(p + ".ffn.project_out", hidden, dim, 1, 1, 1, 0, 1, false));
    if (!ffn_fusable(dim, hidden)) return ZJAI_OK;
    const float *wi, *wd, *wo2;
    ZJAI_TRY(get(p + ".ffn.project_in.weight", {2 * hidden, dim, 1, 1}, &wi));
    ZJAI_TRY(get(p + ".ffn.dwconv.weight", {2 * hidden, 1, 3, 3}, &wd));
    ZJAI_TRY(get(p + ".ffn.project_out.weight", {dim, hidden, 1, 1}, &wo2));
    FfnLayer F;
    ZJAI_TRY(pack_ffn(net->ctx, &F, wi, wd, wo2, dim, hidden));
    net->ffns[p] = F;
    return ZJAI_OK;
  }
  int tam(const std::string& p, int dim, bool ds) {  // Tam::load (attention.rs:509-528)
    if (ds) {
      ZJAI_TRY(conv(p + ".ds_conv", dim, dim, 3, 3, 2, 1, 1, true));
      ZJAI_TRY(convt(p + ".us_conv", dim, dim, 3, 1, 1));
    }
    ZJAI_TRY(tb(p + ".TABs.0", dim));
    return tb(p + ".TABs.1", dim);
  }
  // Upsample::load (synthesis.rs:127-160)
  int upsample(const std::string& prefix, int cin, int cout) {
    if (net->op == ZJAI_BOP) return convt(prefix, cin, cout, 4, 1, 0);
    static const int extra[4] = {0, 0, 1, 1};
    return conv(prefix + ".conv", cin, 4 * cout, 2, 2, 1, 0, 1, false, extra, 2);
  }
};

// eICCI (src/model/icci.rs:64-212): conv `prefix` followed by a per-output-channel affine map
// (an inference-mode batch norm and / or a learned scale), folded into the weights and bias in
// f64 and rounded once, like the crate's `folded_conv`; packed under `store`.
static int icci_fold(Loader& L, const std::string& prefix, const std::string& store, int cin,
                     int cout, int kh, int kw, const std::vector<double>& a,
                     const std::vector<double>& shift) {
  const float *w, *b;
  ZJAI_TRY(L.get(prefix + ".weight", {cout, cin, kh, kw}, &w));
  ZJAI_TRY(L.get(prefix + ".bias", {cout}, &b));
  const size_t per = (size_t)cin * kh * kw;
  std::vector<float> wf((size_t)cout * per), bf(cout);
  for (int o = 0; o < cout; ++o) {
    for (size_t i = 0; i < per; ++i) wf[o * per + i] = (float)((double)w[o * per + i] * a[o]);
    bf[o] = (float)((double)b[o] * a[o] + shift[o]);
  }
  ConvLayer C;
  ZJAI_TRY(pack_conv(L.net->ctx, &C, wf.data(), bf.data(), cin, cout, kh, kw, 1, kh / 2, kw / 2,
                     1, nullptr, 1));
  L.net->convs[store] = C;
  return ZJAI_OK;
}

// a scalar parameter ([] or [1])
static int icci_scalar(Loader& L, const std::string& name, double* out) {
  auto it = L.byname.find(name);
  if (it == L.byname.end()) return fail(ZJAI_MODEL, name + ": missing");
  const zjai_param* p = it->second;
  if (p->ndim > 1 || (p->ndim == 1 && p->shape[0] != 1) || !p->data)
    return fail(ZJAI_MODEL, name + ": not a scalar");
  *out = (double)p->data[0];
  return ZJAI_OK;
}

// batch_norm (icci.rs:64-87): (a s, (beta - mean a) s) with a = gamma / sqrt(var + 1e-5)
static int icci_bn(Loader& L, const std::string& prefix, int ch, double s, std::vector<double>* a,
                   std::vector<double>* shift) {
  const float *g, *be, *m, *v;
  ZJAI_TRY(L.get(prefix + ".weight", {ch}, &g));
  ZJAI_TRY(L.get(prefix + ".bias", {ch}, &be));
  ZJAI_TRY(L.get(prefix + ".running_mean", {ch}, &m));
  ZJAI_TRY(L.get(prefix + ".running_var", {ch}, &v));
  a->resize(ch);
  shift->resize(ch);
  for (int c = 0; c < ch; ++c) {
    const double k = (double)g[c] / std::sqrt((double)v[c] + 1e-5);
    (*a)[c] = k * s;
    (*shift)[c] = ((double)be[c] - (double)m[c] * k) * s;
  }
  return ZJAI_OK;
}

// Trunk::load (icci.rs:137-166): packed as "<tag>.first", "<tag>.<i>.c1", "<tag>.<i>.c2"
static int icci_trunk(Loader& L, const std::string& first, const std::string& bn,
                      const std::string& hidden, int blocks, const std::string& tag) {
  const int nf = kIcciFeatures;
  if (L.has(hidden + "." + std::to_string(blocks) + ".scale"))
    return fail(ZJAI_MODEL, hidden + ": more than " + std::to_string(blocks) + " residual blocks");
  std::vector<double> a, sh, a2, sh2;
  ZJAI_TRY(icci_bn(L, bn, nf, 1.0, &a, &sh));
  ZJAI_TRY(icci_fold(L, first, tag + ".first", 3 * kIcciBands, nf, 3, 3, a, sh));
  for (int i = 0; i < blocks; ++i) {
    const std::string p = hidden + "." + std::to_string(i), q = tag + "." + std::to_string(i);
    double s;
    ZJAI_TRY(icci_scalar(L, p + ".scale", &s));
    ZJAI_TRY(icci_bn(L, p + ".BN1", nf, 1.0, &a, &sh));
    ZJAI_TRY(icci_bn(L, p + ".BN2", nf, s, &a2, &sh2));
    ZJAI_TRY(icci_fold(L, p + ".conv1", q + ".c1", nf, nf, 1, 3, a, sh));
    ZJAI_TRY(icci_fold(L, p + ".conv2", q + ".c2", nf, nf, 3, 1, a2, sh2));
  }
  return ZJAI_OK;
}

static int icci_last(Loader& L, const std::string& conv, const std::string& scale,
                     const std::string& store) {
  double s;
  ZJAI_TRY(icci_scalar(L, scale, &s));
  return icci_fold(L, conv, store, kIcciFeatures, kIcciBands, 3, 3,
                   std::vector<double>(kIcciBands, s), std::vector<double>(kIcciBands, 0.0));
}

static int load_net(Net* n, Loader& L) {
  const int op = n->op;
  switch (n->kind) {
    case ZJAI_SYN_Y:
      if (op == ZJAI_HOP) {  // HopPrimary::load (synthesis.rs:340-354)
        const int c = 128;
        ZJAI_TRY(L.rb("first_stage.0.0", 160));
        ZJAI_TRY(L.convt("first_stage.1", 160, c, 3, 1, 1));
        ZJAI_TRY(L.resau("first_stage.2", c));
        ZJAI_TRY(L.convt("conv2_t", c, c, 3, 1, 1));
        ZJAI_TRY(L.cab("CAB", c));
        ZJAI_TRY(L.resau("iact2", c));
        ZJAI_TRY(L.conv("conv3_t", c, 4 * c, 1, 1, 1, 0, 1, true, nullptr, 2));
        ZJAI_TRY(L.tam("TAM", c, true));
        ZJAI_TRY(L.resau("iact3", c));
        return L.convt("conv4_t", c, 1, 3, 1, 1);
      } else {  // LightPrimary::load (synthesis.rs:521-548)
        const int c1 = 64, c2 = op == ZJAI_SOP ? 32 : 64, c3 = op == ZJAI_SOP ? 32 : 96;
        ZJAI_TRY(L.conv("first_stage.0.0.conv1", 160, 160, 3, 3, 1, 1, 1, true));
        ZJAI_TRY(L.upsample("first_stage.1", 160, c1));
        ZJAI_TRY(L.resau("first_stage.2", c1));
        ZJAI_TRY(L.upsample("conv2_t", c1, c2));
        ZJAI_TRY(L.resau("iact2", c2));
        ZJAI_TRY(L.conv("conv3", c2, c3, 3, 3, 1, 1, 1, true));
        ZJAI_TRY(L.resau("iact3", c3));
        return L.conv("conv4", c3, 16, 1, 1, 1, 0, 1, false, nullptr, 4);
      }
    case ZJAI_SYN_UV:
      ZJAI_TRY(L.conv("first_stage.conv1", 256, 48, 3, 3, 1, 1, 1, true));
      if (op == ZJAI_HOP) {  // HopSecondary::load (synthesis.rs:735-747)
        const int c = 64;
        ZJAI_TRY(L.convt("conv2_t", 144, c, 3, 1, 1));
        ZJAI_TRY(L.cab("CAB", c));
        ZJAI_TRY(L.resau("iact2", c));
        ZJAI_TRY(L.conv("conv3_t", c, 4 * c, 1, 1, 1, 0, 1, true, nullptr, 2));
        ZJAI_TRY(L.tam("TAM", c, false));
        ZJAI_TRY(L.resau("iact3", c));
        return L.convt("conv4_t", c, 8, 3, 1, 1, 2);
      } else {  // LightSecondary::load (synthesis.rs:870-885)
        const int c2 = op == ZJAI_SOP ? 32 : 64, c3 = op == ZJAI_SOP ? 32 : 128;
        ZJAI_TRY(L.upsample("conv2_t", 144, c2));
        ZJAI_TRY(L.resau("iact2", c2));
        ZJAI_TRY(L.conv("conv3", c2, c3, 3, 3, 1, 1, 1, true));
        ZJAI_TRY(L.resau("iact3", c3));
        return L.conv("conv4", c3, 128, 1, 1, 1, 0, 1, false, nullptr, 8);
      }
    case ZJAI_ANA_Y:
    case ZJAI_ANA_UV: {  // Trunk::load + AnalysisPrimary/Secondary::load (analysis.rs:118-289)
      if (op == ZJAI_SOP) return fail(ZJAI_INVALID_ARGUMENT, "there is no SOP analysis transform (use BOP)");
      const bool sec = n->kind == ZJAI_ANA_UV, hop = op == ZJAI_HOP;
      const int c = 128;
      ZJAI_TRY(L.conv("conv1", sec ? 12 : 1, c, 3, 3, 2, 1, 1, true));
      if (!sec) ZJAI_TRY(L.conv_im2col("conv1", c));
      ZJAI_TRY(L.resau("act1", c));
      if (hop) ZJAI_TRY(L.tam("TAM", c, !sec));
      ZJAI_TRY(L.conv("conv2", c, c, 3, 3, 2, 1, 1, true));
      ZJAI_TRY(L.resau("act2", c));
      if (hop) ZJAI_TRY(L.cab("cab", c));
      ZJAI_TRY(L.conv("conv3", c, c, 3, 3, 2, 1, 1, true));
      ZJAI_TRY(L.resau("act3", c));
      if (sec) return L.conv("conv5", c, 96, 1, 1, 1, 0, 1, false);
      ZJAI_TRY(L.conv("conv4", c, 160, 3, 3, 2, 1, 1, true));
      return L.conv("conv5", 160, 160, 1, 1, 1, 0, 1, false);
    }
    case ZJAI_ICCI:  // IcciNet::load (icci.rs:181-212)
      ZJAI_TRY(icci_trunk(L, "conv_first_Y", "BNY", "hidden_layer_Y", kIcciLumaBlocks, "icci.y"));
      ZJAI_TRY(icci_last(L, "conv_last_Y", "scaleY", "icci.last_y"));
      ZJAI_TRY(icci_trunk(L, "conv_firstUV", "BNUV", "hidden_layer_UV", kIcciChromaBlocks,
                          "icci.uv"));
      ZJAI_TRY(icci_last(L, "conv_last_u", "scaleU", "icci.last_u"));
      return icci_last(L, "conv_last_v", "scaleV", "icci.last_v");
    case ZJAI_LATENT: {
      // HyperDecoder::load (hyper_decoder.rs:24-42); ContextModel::load (mcm.rs:119-156) when
      // the checkpoint holds "context.MCM.0.fusion_pred_net.conv1.weight" (common.rs:111-115).
      // The channel count is the checkpoint's (160 luma, 96 chroma in the crate).
      auto it = L.byname.find("hyper_decoder.conv1.weight");
      if (it == L.byname.end() || it->second->ndim != 4)
        return fail(ZJAI_MODEL, "hyper_decoder.conv1.weight: missing or not 4-D");
      const int c = (int)it->second->shape[0];
      if (c <= 0 || c % 16)
        return fail(ZJAI_UNSUPPORTED, "latent networks: channel count must be a multiple of 16");
      n->lat_c = c;
      ZJAI_TRY(L.conv("hyper_decoder.conv1", c, c, 1, 1, 1, 0, 1, false));
      ZJAI_TRY(L.convt("hyper_decoder.conv2", c, c, 4, 1, 0));
      ZJAI_TRY(L.conv("hyper_decoder.conv3", c, c, 3, 3, 1, 1, 1, true));
      ZJAI_TRY(L.conv("hyper_decoder.conv4", c, 4 * c, 3, 3, 1, 1, 1, true));
      if (!L.has("context.MCM.0.fusion_pred_net.conv1.weight")) return ZJAI_OK;
      if (c % 32) return fail(ZJAI_MODEL, "context model: channel count must be a multiple of 32");
      for (int st = 0; st < 4; ++st) {
        const std::string p = "context.MCM." + std::to_string(st);
        if (st > 0) {
          ZJAI_TRY(L.conv(p + ".conv.0", st * c, c, 1, 1, 1, 0, 1, false));
          ZJAI_TRY(L.conv(p + ".conv.1", c, c, 3, 3, 1, 1, c / 32, true));
        }
        const std::string f = p + ".fusion_pred_net";  // FusionPredNet::load (mcm.rs:36-57)
        ZJAI_TRY(L.conv(f + ".conv1", st ? 2 * c : c, c, 1, 1, 1, 0, 1, false));
        ZJAI_TRY(L.conv(f + ".conv2", c, c, 1, 1, 1, 0, 1, false));
        ZJAI_TRY(L.conv(f + ".conv3", c, c, 1, 1, 1, 0, 1, false));
      }
      n->lat_ctx = true;
      return ZJAI_OK;
    }
    default:
      return fail(ZJAI_INVALID_ARGUMENT, "unknown network kind");
  }
}

uint64_t next_net_uid() {
  static std::atomic<uint64_t> next{1};
  return next++;
}

int load_network(Ctx* ctx, int kind, int op, const zjai_param* params, int nparams, Net** out) {
  *out = nullptr;
  // the latent and eICCI networks are the same for every operating point
  if (kind != ZJAI_LATENT && kind != ZJAI_ICCI && (op < ZJAI_SOP || op > ZJAI_HOP))
    return fail(ZJAI_INVALID_ARGUMENT, "unknown operating point");
  if (nparams < 0 || (nparams > 0 && !params)) return fail(ZJAI_INVALID_ARGUMENT, "params");
  Net* n = new Net();
  n->ctx = ctx;
  n->kind = kind;
  n->op = op;
  n->uid = next_net_uid();
  Loader L;
  L.net = n;
  for (int i = 0; i < nparams; ++i) {
    if (!params[i].name) {
      delete n;
      return fail(ZJAI_MODEL, "parameter without a name");
    }
    L.byname[params[i].name] = &params[i];
  }
  int st = load_net(n, L);
  if (st != ZJAI_OK) {
    delete n;
    return st;
  }
  *out = n;
  return ZJAI_OK;
}

// A conv stage composed from the crate's primitives: "conv" (k x k, stride 1, pad k / 2, bias
// optional, `shuffle` folded into its columns) followed by the residual blocks "res.<i>"
// (ResidualBlock::load, attention.rs:22-34) while their parameters are present.
int load_stage(Ctx* ctx, int shuffle, int act, int res_act, const zjai_param* params,
               int nparams, Net** out) {
  *out = nullptr;
  if (shuffle != 1 && shuffle != 2 && shuffle != 4)
    return fail(ZJAI_INVALID_ARGUMENT, "stage: shuffle must be 1, 2 or 4");
  if (act < ACT_NONE || act > ACT_RELU6 || res_act < ACT_NONE || res_act > ACT_RELU6)
    return fail(ZJAI_INVALID_ARGUMENT, "stage: unknown activation");
  if (nparams < 0 || (nparams > 0 && !params)) return fail(ZJAI_INVALID_ARGUMENT, "params");
  std::unique_ptr<Net> n(new Net());
  n->ctx = ctx;
  n->kind = kStageKind;
  n->uid = next_net_uid();
  Loader L;
  L.net = n.get();
  for (int i = 0; i < nparams; ++i) {
    if (!params[i].name) return fail(ZJAI_MODEL, "parameter without a name");
    L.byname[params[i].name] = &params[i];
  }
  auto it = L.byname.find("conv.weight");
  if (it == L.byname.end() || it->second->ndim != 4)
    return fail(ZJAI_MODEL, "conv.weight: missing or not 4-D");
  const int64_t* sh = it->second->shape;
  const int oc = (int)sh[0], cin = (int)sh[1], k = (int)sh[2];
  if (oc <= 0 || cin <= 0 || k <= 0 || sh[3] != k || k % 2 == 0 || oc % (shuffle * shuffle))
    return fail(ZJAI_MODEL, "conv.weight: needs [cout * shuffle^2][cin][k][k] with odd k");
  const int cout = oc / (shuffle * shuffle);
  ZJAI_TRY(L.conv("conv", cin, oc, k, k, 1, k / 2, 1, L.has("conv.bias"), nullptr, shuffle));
  int nres = 0;
  while (L.has("res." + std::to_string(nres) + ".conv1.weight")) {
    ZJAI_TRY(L.rb("res." + std::to_string(nres), cout));
    ++nres;
  }
  n->st_act = act;
  n->st_shuffle = shuffle;
  n->st_res_act = res_act;
  n->st_nres = nres;
  n->st_cin = cin;
  n->st_cout = cout;
  *out = n.release();
  return ZJAI_OK;
}

Net::~Net() {
  for (auto& kv : convs) free_conv(&kv.second);
  for (auto& kv : ffns) free_ffn(&kv.second);
  for (auto& kv : vecs) cudaFree(kv.second);
}

// ---------------------------------------------------------------------------------------------
// Execution
// ---------------------------------------------------------------------------------------------

int Runner::alloc(int h, int w, int c, TView* v) {
  return alloc_tensor(ctx, n, h, w, c, v, false, arena, stream);
}

const ConvLayer* Runner::layer(const std::string& name) {
  auto it = net->convs.find(name);
  return it == net->convs.end() ? nullptr : &it->second;
}

// Profile tag prefix: network kind and batch size ("Y28:" = luma, 28 tiles).
std::string Runner::kind_tag() const {
  static const char* k[] = {"Y", "UV", "AY", "AUV"};
  if (net->kind == ZJAI_LATENT) return "L" + std::to_string(net->lat_c) + ":";
  if (net->kind == ZJAI_ICCI) return "I:";
  if (net->kind == kStageKind) return "S" + std::to_string(n) + ":";
  return std::string(k[net->kind & 3]) + std::to_string(n) + ":";
}

int Runner::conv(const std::string& name, const TView& in, ConvOut o) {
  const ConvLayer* L = layer(name);
  if (!L) return fail(ZJAI_MODEL, name + ": layer not loaded");
  return conv_layer(name, *L, in, o);
}

int Runner::conv_layer(const std::string& name, const ConvLayer& layer_ref, const TView& in,
                       ConvOut o) {
  const ConvLayer* L = &layer_ref;
  cudaStream_t saved = ctx->stream;
  ctx->stream = stream;
  ctx->cur_arena = arena;
  if (ctx->profiling) ctx->tag = kind_tag() + name;
  int st = run_conv(ctx, *L, in, o);
  ctx->stream = saved;
  ctx->cur_arena = nullptr;
  if (st == ZJAI_OK && count_flops) {
    int oh, ow, out_h, out_w;
    L->out_size(in.h, in.w, &oh, &ow, &out_h, &out_w);
    const int wh = o.planar ? (o.out_h >= 0 ? o.out_h : out_h) : o.out.h;
    const int ww = o.planar ? (o.out_w >= 0 ? o.out_w : out_w) : o.out.w;
    oh = std::min(oh, cdiv(wh, L->R));
    ow = std::min(ow, cdiv(ww, L->R));
    flops += (double)L->flops_per_px * oh * ow * in.n;
  }
  return st;
}

// Output extent of a layer for an input of h x w.
int Runner::out_extent(const std::string& name, int h, int w, int* oh, int* ow) {
  const ConvLayer* L = layer(name);
  if (!L) return fail(ZJAI_MODEL, name + ": layer not loaded");
  int a, b;
  L->out_size(h, w, &a, &b, oh, ow);
  return ZJAI_OK;
}

int Runner::stop_check() {
  if (cancel && *cancel) return fail(ZJAI_CANCELLED, "stopped: cancelled by the caller");
  return ZJAI_OK;
}

int Runner::probe(const char* name, const TView& t) {
  if (ctx->probes.empty()) return ZJAI_OK;
  auto it = ctx->probes.find(name);
  if (it == ctx->probes.end()) return ZJAI_OK;
  if ((long long)t.n * t.c * t.h * t.w > it->second.second)
    return fail(ZJAI_LIMIT_EXCEEDED, std::string("probe ") + name + ": buffer too small");
  float* dst = it->second.first;
  mem_kernel(std::string("probe.") + name, "copy", (double)t.n * t.c * t.h * t.w * 6.0, 1,
             [&] { launch_nhwc_to_planar(t, dst, stream); });
  return cuda_check(cudaGetLastError(), "probe");
}

// ResAu::forward (synthesis.rs:61-74): y = x * (1 + conv1x1(gconv3x3(relu6 x))), cropped to
// (ch, cw) afterwards (the reference's crop follows the block). `a` = relu6(x).
int Runner::resau(const std::string& p, const TView& x, const TView& a, int ch, int cw,
                  TView* y) {
  ArenaMark mark(arena);
  TView t;
  ZJAI_TRY(alloc(ch, cw, x.c, &t));
  ConvOut o1;
  o1.out = t;
  ZJAI_TRY(conv(p + ".conv", a, o1));
  TView xc = x.crop(ch, cw);
  ConvOut o2;
  o2.out = xc;
  o2.op = OP_GATE;
  o2.r1 = &xc;
  ZJAI_TRY(conv(p + ".conv2", t, o2));  // in place: each element reads x then writes y
  *y = xc;
  return ZJAI_OK;
}

// ResidualBlock::forward (attention.rs:36-43): conv2(relu(conv1 x)) + x -> *y (may alias x).
// `act` replaces the ReLU between the convs (LeakyReLU in the conv stages of BASELINE configs).
int Runner::rb(const std::string& p, const TView& x, const TView& y, const TView* relu6_out,
               int act) {
  ArenaMark mark(arena);
  TView t;
  ZJAI_TRY(alloc(x.h, x.w, x.c, &t));
  ConvOut o1;
  o1.out = t;
  o1.act1 = act;
  ZJAI_TRY(conv(p + ".conv1", x, o1));
  ConvOut o2;
  o2.out = y;
  o2.op = OP_ADD;
  o2.r1 = &x;
  o2.out2 = relu6_out;
  return conv(p + ".conv2", t, o2);
}

// Cab::forward (attention.rs:122-139): x + RB(RB(x)) * sigmoid(convT(RB(RB(conv_s2 x)))),
// written into `out` (a crop of the natural extent), with relu6(out) into `a_out`.
int Runner::cab(const std::string& p, const TView& x, const TView& out, const TView* a_out) {
  if ((x.h & 1) || (x.w & 1)) return fail(ZJAI_INVALID_ARGUMENT, "CAB: odd feature map size");
  ArenaMark mark(arena);
  TView tr;
  ZJAI_TRY(alloc(x.h, x.w, x.c, &tr));
  ZJAI_TRY(rb(p + ".residual_trunk.0", x, tr));
  ZJAI_TRY(rb(p + ".residual_trunk.1", tr, tr));
  int mh, mw;
  ZJAI_TRY(out_extent(p + ".subscale", x.h, x.w, &mh, &mw));
  TView m;
  ZJAI_TRY(alloc(mh, mw, x.c, &m));
  ConvOut os;
  os.out = m;
  ZJAI_TRY(conv(p + ".subscale", x, os));
  ZJAI_TRY(rb(p + ".residual_mask2.0", m, m));
  ZJAI_TRY(rb(p + ".residual_mask3.0", m, m));
  const TView trc = tr.crop(out.h, out.w), xc = x.crop(out.h, out.w);
  ConvOut ou;
  ou.out = out;
  ou.act1 = ACT_SIGMOID;
  ou.op = OP_CAB;
  ou.r1 = &trc;
  ou.r2 = &xc;
  ou.out2 = a_out;
  return conv(p + ".upscale", m, ou);
}

// TransformerBlock::forward (attention.rs:328-372), in place on x.
int Runner::tb(const std::string& p, const TView& x) {
  const int d = x.c, hidden = 4 * d;
  auto vec = [&](const std::string& k) { return net->vecs.at(k); };
  ArenaMark mark(arena);
  TView ln, qkv, qkv2;
  ZJAI_TRY(alloc(x.h, x.w, d, &ln));
  ZJAI_TRY(alloc(x.h, x.w, 3 * d, &qkv));
  ZJAI_TRY(alloc(x.h, x.w, 3 * d, &qkv2));
  // algorithmic bytes per pixel of a d-channel f16 map
  const double px = (double)n * x.h * x.w, b16 = 2.0 * px;
  mem_kernel(p + ".prep_data.norm1", "ln", 2 * b16 * d, 1, [&] {
    launch_layer_norm(x, ln, vec(p + ".prep_data.norm1.weight"),
                      vec(p + ".prep_data.norm1.bias"), stream);
  });
  ConvOut o;
  o.out = qkv;
  ZJAI_TRY(conv(p + ".prep_data.conv1", ln, o));
  int st = ZJAI_OK;
  mem_kernel(p + ".prep_data.conv2", "dw", 2 * b16 * 3 * d, 1, [&] {
    st = launch_dw3x3(ctx, qkv, qkv2, vec(p + ".prep_data.conv2"), false, stream);
  });
  ZJAI_TRY(st);
  float* scratch = static_cast<float*>(
      arena->alloc(attention_scratch_floats(n, d, 4, x.h * x.w, ctx->sms) * sizeof(float)));
  if (!scratch) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (attention scratch)");
  // x += W_o (A . v): the attention matrices A_n, folded into per-picture projection weights
  // W_o . blockdiag(A_n), then one tcgen05 1x1 conv over the v slice of qkv2. The Gram reads
  // q and k; the conv reads v.
  const ConvLayer* Lo = layer(p + ".attn.project_out");
  if (!Lo) return fail(ZJAI_MODEL, p + ".attn.project_out: layer not loaded");
  const long long wset = (long long)Lo->npad * Lo->cin_pad;
  __half* wfold = static_cast<__half*>(arena->alloc((size_t)n * wset * sizeof(__half)));
  if (!wfold) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (folded weights)");
  const float fs = net->fold_scale.at(p);
  mem_kernel(p + ".attn", "attn", b16 * 2 * d, attention_fold_launches(d, 4, *Lo), [&] {
    launch_attention_fold(qkv2, 4, vec(p + ".attn.temperature"),
                          vec(p + ".attn.project_out.weight"), fs, *Lo, wfold, scratch, ctx->sms,
                          stream);
  });
  if (count_flops) flops += 2.0 * 2.0 * (double)n * x.h * x.w * d * (d / 4);
  ConvLayer Lf = *Lo;
  Lf.w = wfold;
  Lf.w_img = wset;
  Lf.klist = nullptr;  // W_o . blockdiag(A) has its own zero pattern: run every K step
  Lf.koff = nullptr;
  Lf.scale = 1.f / fs;
  ConvOut oa;
  oa.out = x;
  oa.op = OP_ADD;
  oa.r1 = &x;
  ZJAI_TRY(conv_layer(p + ".attn.project_out", Lf, qkv2.channels(2 * d, d), oa));
  mem_kernel(p + ".ffn.norm1", "ln", 2 * b16 * d, 1, [&] {
    launch_layer_norm(x, ln, vec(p + ".ffn.norm1.weight"), vec(p + ".ffn.norm1.bias"), stream);
  });
  auto fz = net->ffns.find(p);
  if (fz != net->ffns.end()) {
    // project_in, depthwise + gate and project_out in one kernel (ffn_tc.cu)
    cudaStream_t saved = ctx->stream;
    ctx->stream = stream;
    if (ctx->profiling) ctx->tag = kind_tag() + p + ".ffn[fused]";
    st = run_ffn(ctx, fz->second, ln, x);
    ctx->stream = saved;
    if (st == ZJAI_OK && count_flops)
      flops += 2.0 * px * 3.0 * hidden * d;
    return st;
  }
  TView f, g;
  ZJAI_TRY(alloc(x.h, x.w, 2 * hidden, &f));
  ZJAI_TRY(alloc(x.h, x.w, hidden, &g));
  ConvOut oi;
  oi.out = f;
  ZJAI_TRY(conv(p + ".ffn.project_in", ln, oi));
  mem_kernel(p + ".ffn.dwconv", "dw", b16 * 3 * hidden, 1, [&] {
    st = launch_dw3x3(ctx, f, g, vec(p + ".ffn.dwconv"), true, stream);
  });
  ZJAI_TRY(st);
  ConvOut of;
  of.out = x;
  of.op = OP_ADD;
  of.r1 = &x;
  return conv(p + ".ffn.project_out", g, of);
}

// Tam::forward (attention.rs:530-545). Without resampling the blocks run in place on x and
// *y = x cropped; with resampling the output goes into a new map of extent (ch, cw).
int Runner::tam(const std::string& p, const TView& x, bool ds, int ch, int cw, TView* y,
                TView* a_out) {
  if (!ds) {
    ZJAI_TRY(tb(p + ".TABs.0", x));
    ZJAI_TRY(tb(p + ".TABs.1", x));
    *y = x.crop(ch, cw);
    TView a;
    ZJAI_TRY(alloc(ch, cw, x.c, &a));
    launch_relu6(*y, a, stream);
    ctx->launches++;
    *a_out = a;
    return ZJAI_OK;
  }
  int th, tw;
  ZJAI_TRY(out_extent(p + ".ds_conv", x.h, x.w, &th, &tw));
  TView t;
  ZJAI_TRY(alloc(th, tw, x.c, &t));
  ConvOut od;
  od.out = t;
  ZJAI_TRY(conv(p + ".ds_conv", x, od));
  ZJAI_TRY(tb(p + ".TABs.0", t));
  ZJAI_TRY(tb(p + ".TABs.1", t));
  TView o, a;
  ZJAI_TRY(alloc(ch, cw, x.c, &o));
  ZJAI_TRY(alloc(ch, cw, x.c, &a));
  ConvOut ou;
  ou.out = o;
  ou.out2 = &a;
  ZJAI_TRY(conv(p + ".us_conv", t, ou));
  *y = o;
  *a_out = a;
  return ZJAI_OK;
}

// Upsample::forward (synthesis.rs:162-171) into a map of extent (ch, cw), relu6 copy in a_out.
int Runner::upsample(const std::string& p, const TView& x, int ch, int cw, TView* y,
                     TView* a_out) {
  const std::string name = net->op == ZJAI_BOP ? p : p + ".conv";
  const ConvLayer* L = layer(name);
  if (!L) return fail(ZJAI_MODEL, name + ": layer not loaded");
  const int c = L->cph;  // output channels (the shuffle folds the rest into pixels)
  ZJAI_TRY(alloc(ch, cw, c, y));
  ZJAI_TRY(alloc(ch, cw, c, a_out));
  ConvOut o;
  o.out = *y;
  o.out2 = a_out;
  return conv(name, x, o);
}

// Final planar output of a synthesis network.
int Runner::final_planar(const std::string& name, const TView& x, const FinalOut& fo) {
  ConvOut o;
  o.planar = true;
  o.denorm = true;
  o.clamp = ctx->clamp_output;
  o.pout = fo.plane0;
  o.pout2 = fo.plane1;
  o.p_plane = fo.plane_stride;
  o.p_row = fo.row;
  o.p_img = fo.img;
  o.img_win = fo.win;
  o.sv = fo.sv;
  o.sh = fo.sh;
  o.qbytes = fo.qbytes;
  o.qmax = fo.qmax;
  if (fo.full_h > 0) {
    o.out_h = fo.full_h;
    o.out_w = fo.full_w;
  }
  return conv(name, x, o);
}

// LightPrimary::forward (synthesis.rs:550-580) / HopPrimary::forward (:356-390) on a batch of
// latents y [n][lh][lw][>=160] for tiles of h x w samples.
int Runner::primary(const TView& y, int h, int w, const FinalOut& fo) {
  const int op = net->op;
  if (y.c != 160) return fail(ZJAI_INVALID_ARGUMENT, "primary: latent must have 160 channels");
  const int h8 = cdiv(h, 8), w8 = cdiv(w, 8), h4 = cdiv(h, 4), w4 = cdiv(w, 4);
  const int h2 = cdiv(h, 2), w2 = cdiv(w, 2);
  if (2 * y.h < h8 || 2 * y.w < w8) return fail(ZJAI_INVALID_ARGUMENT, "crop larger than tensor");
  if (op != ZJAI_HOP) {
    TView x0;
    ZJAI_TRY(alloc(y.h, y.w, 160, &x0));
    ConvOut o;
    o.out = x0;
    o.act1 = ACT_RELU;
    o.op = OP_ADD;
    o.r1 = &y;
    ZJAI_TRY(conv("first_stage.0.0.conv1", y, o));
    ZJAI_TRY(stop_check());
    TView x1, a1;
    ZJAI_TRY(upsample("first_stage.1", x0, 2 * y.h, 2 * y.w, &x1, &a1));
    TView x1c;
    ZJAI_TRY(resau("first_stage.2", x1, a1, h8, w8, &x1c));
    ZJAI_TRY(stop_check());
    if (2 * h8 < h4 || 2 * w8 < w4) return fail(ZJAI_INVALID_ARGUMENT, "crop larger than tensor");
    TView x2, a2;
    ZJAI_TRY(upsample("conv2_t", x1c, h4, w4, &x2, &a2));
    ZJAI_TRY(stop_check());
    TView x2c;
    ZJAI_TRY(resau("iact2", x2, a2, h4, w4, &x2c));
    ZJAI_TRY(stop_check());
    const ConvLayer* c3 = layer("conv3");
    TView x3, a3;
    ZJAI_TRY(alloc(h4, w4, c3->cph, &x3));
    ZJAI_TRY(alloc(h4, w4, c3->cph, &a3));
    ConvOut o3;
    o3.out = x3;
    o3.out2 = &a3;
    ZJAI_TRY(conv("conv3", x2c, o3));
    ZJAI_TRY(stop_check());
    TView x3c;
    ZJAI_TRY(resau("iact3", x3, a3, h4, w4, &x3c));
    ZJAI_TRY(stop_check());
    return final_planar("conv4", x3c, fo);
  }
  // HOP
  TView x0;
  ZJAI_TRY(alloc(y.h, y.w, 160, &x0));
  ZJAI_TRY(rb("first_stage.0.0", y, x0));
  ZJAI_TRY(stop_check());
  TView x1, a1;
  ZJAI_TRY(alloc(2 * y.h, 2 * y.w, 128, &x1));
  ZJAI_TRY(alloc(2 * y.h, 2 * y.w, 128, &a1));
  {
    ConvOut o;
    o.out = x1;
    o.out2 = &a1;
    ZJAI_TRY(conv("first_stage.1", x0, o));
  }
  TView x1c;
  ZJAI_TRY(resau("first_stage.2", x1, a1, h8, w8, &x1c));
  ZJAI_TRY(stop_check());
  TView x2;
  ZJAI_TRY(alloc(2 * h8, 2 * w8, 128, &x2));
  {
    ConvOut o;
    o.out = x2;
    ZJAI_TRY(conv("conv2_t", x1c, o));
  }
  if (2 * h8 < h4 || 2 * w8 < w4) return fail(ZJAI_INVALID_ARGUMENT, "crop larger than tensor");
  TView xc, ac;
  ZJAI_TRY(alloc(h4, w4, 128, &xc));
  ZJAI_TRY(alloc(h4, w4, 128, &ac));
  ZJAI_TRY(cab("CAB", x2, xc, &ac));
  ZJAI_TRY(stop_check());
  TView x2c;
  ZJAI_TRY(resau("iact2", xc, ac, h4, w4, &x2c));
  ZJAI_TRY(stop_check());
  TView x3;
  ZJAI_TRY(alloc(2 * h4, 2 * w4, 128, &x3));
  {
    ConvOut o;
    o.out = x3;
    ZJAI_TRY(conv("conv3_t", x2c, o));
  }
  ZJAI_TRY(stop_check());
  TView xt, at;
  ZJAI_TRY(tam("TAM", x3, true, h2, w2, &xt, &at));
  ZJAI_TRY(stop_check());
  TView x4;
  ZJAI_TRY(resau("iact3", xt, at, h2, w2, &x4));
  ZJAI_TRY(stop_check());
  return final_planar("conv4_t", x4, fo);
}

// SynthesisSecondary::forward_with (synthesis.rs:1004-1038): `cat` holds the luma latent
// (channels 0..159, cropped to the chroma latent) and the chroma latent (160..255); `x144`
// already holds the chroma latent in channels 48..143.
int Runner::secondary(const TView& cat, const TView& x144, int h, int w, const FinalOut& fo) {
  const int op = net->op;
  if (cat.c != 256 || x144.c != 144) return fail(ZJAI_INVALID_ARGUMENT, "secondary: latent channels");
  {
    ConvOut o;
    o.out = x144.channels(0, 48);
    ZJAI_TRY(conv("first_stage.conv1", cat, o));
  }
  ZJAI_TRY(stop_check());
  const int h8 = cdiv(h, 8), w8 = cdiv(w, 8), h4 = cdiv(h, 4), w4 = cdiv(w, 4);
  if (2 * cat.h < h8 || 2 * cat.w < w8) return fail(ZJAI_INVALID_ARGUMENT, "crop larger than tensor");
  if (op != ZJAI_HOP) {
    TView x1, a1;
    ZJAI_TRY(upsample("conv2_t", x144, h8, w8, &x1, &a1));
    ZJAI_TRY(stop_check());
    TView x1c;
    ZJAI_TRY(resau("iact2", x1, a1, h8, w8, &x1c));
    ZJAI_TRY(stop_check());
    const ConvLayer* c3 = layer("conv3");
    TView x3, a3;
    ZJAI_TRY(alloc(h8, w8, c3->cph, &x3));
    ZJAI_TRY(alloc(h8, w8, c3->cph, &a3));
    ConvOut o3;
    o3.out = x3;
    o3.out2 = &a3;
    ZJAI_TRY(conv("conv3", x1c, o3));
    ZJAI_TRY(stop_check());
    TView x3c;
    ZJAI_TRY(resau("iact3", x3, a3, h8, w8, &x3c));
    ZJAI_TRY(stop_check());
    return final_planar("conv4", x3c, fo);
  }
  const int c = 64;
  TView x1;
  ZJAI_TRY(alloc(2 * cat.h, 2 * cat.w, c, &x1));
  {
    ConvOut o;
    o.out = x1;
    ZJAI_TRY(conv("conv2_t", x144, o));
  }
  TView xc, ac;
  ZJAI_TRY(alloc(h8, w8, c, &xc));
  ZJAI_TRY(alloc(h8, w8, c, &ac));
  ZJAI_TRY(cab("CAB", x1, xc, &ac));
  ZJAI_TRY(stop_check());
  TView x2c;
  ZJAI_TRY(resau("iact2", xc, ac, h8, w8, &x2c));
  ZJAI_TRY(stop_check());
  TView x3;
  ZJAI_TRY(alloc(2 * h8, 2 * w8, c, &x3));
  {
    ConvOut o;
    o.out = x3;
    ZJAI_TRY(conv("conv3_t", x2c, o));
  }
  ZJAI_TRY(stop_check());
  if (2 * h8 < h4 || 2 * w8 < w4) return fail(ZJAI_INVALID_ARGUMENT, "crop larger than tensor");
  TView xt, at;
  ZJAI_TRY(tam("TAM", x3, false, h4, w4, &xt, &at));
  ZJAI_TRY(stop_check());
  TView x4;
  ZJAI_TRY(resau("iact3", xt, at, h4, w4, &x4));
  ZJAI_TRY(stop_check());
  return final_planar("conv4_t", x4, fo);
}

// Trunk::forward (analysis.rs:157-206) + AnalysisPrimary/Secondary heads on a batch of
// normalised, replicate-padded inputs. Output planar f32 [n][C][oh][ow].
int Runner::analysis(const TView& x, int h, int w, float* out) {
  const bool sec = net->kind == ZJAI_ANA_UV, hop = net->op == ZJAI_HOP;
  auto padded = [&](int d) { return 2 * cdiv(h, 2 * d); };
  auto paddedw = [&](int d) { return 2 * cdiv(w, 2 * d); };
  // conv1 on the padded input (h1 = ceil(h/2) etc.)
  int h1 = cdiv(h, 2), w1 = cdiv(w, 2);
  TView x1, a1;
  // allocated at the padded extent so the replicate pad can be written in place
  ZJAI_TRY(alloc(padded(2), paddedw(2), 128, &x1));
  ZJAI_TRY(alloc(padded(2), paddedw(2), 128, &a1));
  x1 = x1.crop(h1, w1);
  a1 = a1.crop(h1, w1);
  {
    ConvOut o;
    o.out = x1;
    o.out2 = &a1;
    // x with 9 channels: the input already laid out as conv1's taps per output pixel
    // (launch_normalize_im2col), for the 1x1 form of conv1
    ZJAI_TRY(conv(x.c == 9 ? "conv1#im2col" : "conv1", x, o));
  }
  TView y1;
  ZJAI_TRY(resau("act1", x1, a1, h1, w1, &y1));
  ZJAI_TRY(probe("ana.act1", y1));
  ZJAI_TRY(stop_check());
  TView p1 = y1.crop(padded(2), paddedw(2));
  launch_replicate_pad(y1, p1, stream);
  ctx->launches++;
  if (hop) {
    TView t, a;
    ZJAI_TRY(tam("TAM", p1, !sec, p1.h, p1.w, &t, &a));
    p1 = t;
  }
  int h2 = cdiv(h, 4), w2 = cdiv(w, 4);
  TView x2, a2;
  ZJAI_TRY(alloc(padded(4), paddedw(4), 128, &x2));
  ZJAI_TRY(alloc(padded(4), paddedw(4), 128, &a2));
  x2 = x2.crop(h2, w2);
  a2 = a2.crop(h2, w2);
  {
    ConvOut o;
    o.out = x2;
    o.out2 = &a2;
    ZJAI_TRY(conv("conv2", p1, o));
  }
  TView y2;
  ZJAI_TRY(resau("act2", x2, a2, h2, w2, &y2));
  ZJAI_TRY(probe("ana.act2", y2));
  ZJAI_TRY(stop_check());
  TView p2 = y2.crop(padded(4), paddedw(4));
  launch_replicate_pad(y2, p2, stream);
  ctx->launches++;
  if (hop) {
    TView c2;
    ZJAI_TRY(alloc(p2.h, p2.w, 128, &c2));
    ZJAI_TRY(cab("cab", p2, c2, nullptr));
    p2 = c2;
  }
  int h3 = cdiv(h, 8), w3 = cdiv(w, 8);
  TView x3, a3;
  ZJAI_TRY(alloc(padded(8), paddedw(8), 128, &x3));
  ZJAI_TRY(alloc(padded(8), paddedw(8), 128, &a3));
  x3 = x3.crop(h3, w3);
  a3 = a3.crop(h3, w3);
  {
    ConvOut o;
    o.out = x3;
    o.out2 = &a3;
    ZJAI_TRY(conv("conv3", p2, o));
  }
  TView y3;
  ZJAI_TRY(resau("act3", x3, a3, h3, w3, &y3));
  ZJAI_TRY(probe("ana.act3", y3));
  ZJAI_TRY(stop_check());
  ConvOut of;
  of.planar = true;
  of.pout = out;
  if (sec) {
    of.p_plane = (long long)h3 * w3;
    of.p_row = w3;
    of.p_img = 96LL * h3 * w3;
    return conv("conv5", y3, of);
  }
  TView p3 = y3.crop(padded(8), paddedw(8));
  launch_replicate_pad(y3, p3, stream);
  ctx->launches++;
  const int h4 = cdiv(h, 16), w4 = cdiv(w, 16);
  TView x4;
  ZJAI_TRY(alloc(h4, w4, 160, &x4));
  {
    ConvOut o;
    o.out = x4;
    ZJAI_TRY(conv("conv4", p3, o));
  }
  of.p_plane = (long long)h4 * w4;
  of.p_row = w4;
  of.p_img = 160LL * h4 * w4;
  return conv("conv5", x4, of);
}

// Conv stage: the first conv (activation, pixel shuffle in its epilogue), then the residual
// blocks in place. Without residual blocks the conv's epilogue writes the planar output.
int Runner::stage(const TView& x, float* out) {
  const ConvLayer* L0 = layer("conv");
  if (!L0) return fail(ZJAI_MODEL, "conv: layer not loaded");
  int oh, ow;
  ZJAI_TRY(out_extent("conv", x.h, x.w, &oh, &ow));
  const int c = net->st_cout;
  if (net->st_nres == 0) {
    ConvOut o;
    o.act1 = net->st_act;
    o.planar = true;
    o.pout = out;
    o.p_plane = (long long)oh * ow;
    o.p_row = ow;
    o.p_img = (long long)c * oh * ow;
    return conv("conv", x, o);
  }
  TView y;
  ZJAI_TRY(alloc(oh, ow, c, &y));
  ConvOut o;
  o.out = y;
  o.act1 = net->st_act;
  ZJAI_TRY(conv("conv", x, o));
  for (int i = 0; i < net->st_nres; ++i) {
    ZJAI_TRY(stop_check());
    ZJAI_TRY(rb("res." + std::to_string(i), y, y, nullptr, net->st_res_act));
  }
  launch_nhwc_to_planar(y, out, stream);
  ctx->launches++;
  return cuda_check(cudaGetLastError(), "nhwc_to_planar");
}

// IcciNet::luma_correction / chroma_corrections (icci.rs:214-241) on the 48 sub-bands x
// (NHWC f16, quarter resolution): trunk(x) = blocks(relu(first(x))), block(f) = f + c2(relu(c1(f)))
// (batch norms and scales folded), then the last convs into planar f32 corrections [16][h][w]
// (null: not wanted). chroma selects the chroma trunk (corrections u, v) instead of luma (y).
int Runner::icci(const TView& x, bool chroma, float* c0, float* c1) {
  const std::string t = chroma ? "icci.uv" : "icci.y";
  const int blocks = chroma ? kIcciChromaBlocks : kIcciLumaBlocks;
  TView f, o;
  ZJAI_TRY(alloc(x.h, x.w, kIcciFeatures, &f));
  ZJAI_TRY(alloc(x.h, x.w, kIcciFeatures, &o));
  {
    ConvOut a;
    a.out = f;
    a.act1 = ACT_RELU;
    ZJAI_TRY(conv(t + ".first", x, a));
  }
  for (int i = 0; i < blocks; ++i) {
    const std::string q = t + "." + std::to_string(i);
    ConvOut a;
    a.out = o;
    a.act1 = ACT_RELU;
    ZJAI_TRY(conv(q + ".c1", f, a));
    ConvOut b;
    b.out = f;
    b.op = OP_ADD;
    b.r1 = &f;
    ZJAI_TRY(conv(q + ".c2", o, b));
  }
  const char* last[2] = {chroma ? "icci.last_u" : "icci.last_y", "icci.last_v"};
  float* dst[2] = {c0, c1};
  for (int k = 0; k < 2; ++k) {
    if (!dst[k]) continue;
    ConvOut a;
    a.planar = true;
    a.pout = dst[k];
    a.p_plane = (long long)x.h * x.w;
    a.p_row = x.w;
    a.p_img = (long long)kIcciBands * x.h * x.w;
    ZJAI_TRY(conv(last[k], f, a));
  }
  return ZJAI_OK;
}

// HyperDecoder::forward_f32 (hyper_decoder.rs:94-113): conv1 1x1 -> convT 4x4 s2, its output
// cropped to (out_h, out_w) with ReLU6 in the epilogue -> conv3 3x3 + ReLU6 -> conv4 3x3 into
// planar f32 psi.
int Runner::hyper(const TView& z, int out_h, int out_w, float* psi) {
  const int c = net->lat_c;
  int nh, nw;
  ZJAI_TRY(out_extent("hyper_decoder.conv2", z.h, z.w, &nh, &nw));
  if (out_h <= 0 || out_w <= 0 || out_h > nh || out_w > nw)
    return fail(ZJAI_INVALID_ARGUMENT, "hyper-decoder: crop larger than the upsampled map");
  TView x1, x2, x3;
  ZJAI_TRY(alloc(z.h, z.w, c, &x1));
  {
    ConvOut o;
    o.out = x1;
    ZJAI_TRY(conv("hyper_decoder.conv1", z, o));
  }
  ZJAI_TRY(alloc(out_h, out_w, c, &x2));
  {
    ConvOut o;
    o.out = x2;
    o.act1 = ACT_RELU6;
    ZJAI_TRY(conv("hyper_decoder.conv2", x1, o));
  }
  ZJAI_TRY(stop_check());
  ZJAI_TRY(alloc(out_h, out_w, c, &x3));
  {
    ConvOut o;
    o.out = x3;
    o.act1 = ACT_RELU6;
    ZJAI_TRY(conv("hyper_decoder.conv3", x2, o));
  }
  ZJAI_TRY(stop_check());
  ConvOut o;
  o.planar = true;
  o.pout = psi;
  o.p_plane = (long long)out_h * out_w;
  o.p_row = out_w;
  o.p_img = 4LL * c * out_h * out_w;
  return conv("hyper_decoder.conv4", x3, o);
}

// The latent from psi and the residual (reconstruct.rs:200-212). With the context model,
// ContextModel::decompress (mcm.rs:161-257) on NHWC f16 maps at half resolution:
//   J   [hh][hw][8C]: stage s's fusion input cat(t_s, psi_s) at channels [2sC, 2sC + 2C)
//                     (psi_s copied in once, t_s written by the stage's grouped conv);
//   ctx [hh][hw][3C]: the reconstructed stages 0..2 (the spatial context), stage s at sC;
// stage s: conv.0 1x1 (sC -> C) on ctx[0, sC) -> conv.1 3x3 grouped into J -> FusionPredNet
// (1x1, ReLU, 1x1, ReLU, 1x1) with the mean as planar f32 -> mcm_stage (mean + residual into
// y_hat and ctx).
int Runner::latent(const float* psi, const float* res, int h, int w, float* y) {
  const int c = net->lat_c;
  if (!net->lat_ctx) {
    mem_kernel("upshuffle", "add", (double)c * h * w * 12.0, 1,
               [&] { launch_upshuffle_add(psi, res, c, h, w, y, stream); });
    return cuda_check(cudaGetLastError(), "upshuffle_psi");
  }
  const int hh = cdiv(h, 2), hw = cdiv(w, 2);
  const double q = (double)c * hh * hw;
  TView J, cx, t0, f1, f2;
  ZJAI_TRY(alloc(hh, hw, 8 * c, &J));
  ZJAI_TRY(alloc(hh, hw, 3 * c, &cx));
  ZJAI_TRY(alloc(hh, hw, c, &t0));
  ZJAI_TRY(alloc(hh, hw, c, &f1));
  ZJAI_TRY(alloc(hh, hw, c, &f2));
  float* mean = static_cast<float*>(arena->alloc((size_t)c * hh * hw * sizeof(float)));
  if (!mean) return fail(ZJAI_LIMIT_EXCEEDED, "device arena exhausted (context model)");
  mem_kernel("psi", "joined", q * 4 * 6.0, 1,
             [&] { launch_psi_to_joined(psi, c, hh, hw, J, stream); });
  static const int PY[4] = {0, 1, 0, 1}, PX[4] = {0, 1, 1, 0};  // mcm.rs:25
  for (int st = 0; st < 4; ++st) {
    ZJAI_TRY(stop_check());
    const std::string p = "context.MCM." + std::to_string(st);
    TView fin = J.channels(c, c);
    if (st > 0) {
      ConvOut o0;
      o0.out = t0;
      ZJAI_TRY(conv(p + ".conv.0", cx.channels(0, st * c), o0));
      ConvOut o1;
      o1.out = J.channels(2 * st * c, c);
      ZJAI_TRY(conv(p + ".conv.1", t0, o1));
      fin = J.channels(2 * st * c, 2 * c);
    }
    ConvOut a1;
    a1.out = f1;
    a1.act1 = ACT_RELU;
    ZJAI_TRY(conv(p + ".fusion_pred_net.conv1", fin, a1));
    ConvOut a2;
    a2.out = f2;
    a2.act1 = ACT_RELU;
    ZJAI_TRY(conv(p + ".fusion_pred_net.conv2", f1, a2));
    ConvOut a3;
    a3.planar = true;
    a3.pout = mean;
    a3.p_plane = (long long)hh * hw;
    a3.p_row = hw;
    a3.p_img = (long long)c * hh * hw;
    ZJAI_TRY(conv(p + ".fusion_pred_net.conv3", f2, a3));
    const TView cs = cx.channels(st * c, c);
    mem_kernel("stage" + std::to_string(st), "mcm", q * (st < 3 ? 14.0 : 12.0), 1, [&] {
      launch_mcm_stage(mean, res, c, h, w, PY[st], PX[st], y, st < 3 ? &cs : nullptr, stream);
    });
  }
  return cuda_check(cudaGetLastError(), "context model");
}

// ---------------------------------------------------------------------------------------------
// Tiling (src/tools/tiles.rs:39-119, 220-229), no independent regions
// ---------------------------------------------------------------------------------------------

int synthesis_tiles(int height, int width, int latent_h, int latent_w, int tile_size,
                    int overlap, std::vector<zjai_tile>* out) {
  out->clear();
  if (height <= 0 || width <= 0) return fail(ZJAI_INVALID_ARGUMENT, "empty picture");
  if (tile_size <= 0) {
    zjai_tile t{0, 0, width, height, 0, 0, latent_w, latent_h, 0, 0, width, height, 0, 0};
    out->push_back(t);
    return ZJAI_OK;
  }
  const int tile_h = std::min(tile_size, height), tile_w = std::min(tile_size, width);
  const int half = overlap / 2;
  if (tile_h <= overlap || tile_w <= overlap)
    return fail(ZJAI_INVALID_DATA, "synthesis tile not larger than its overlap");
  auto extent = [&](int pos, int len, int lat_len, int* r) {
    if (len % 16 && cdiv(pos + len, 16) < lat_len)
      return fail(ZJAI_INVALID_DATA, "unaligned synthesis tile inside the picture");
    *r = cdiv(len, 16);
    return (int)ZJAI_OK;
  };
  for (int y = 0; y < height - overlap; y += tile_h - overlap)
    for (int x = 0; x < width - overlap; x += tile_w - overlap) {
      zjai_tile t;
      t.img_x = x;
      t.img_y = y;
      t.img_w = std::min(tile_w, width - x);
      t.img_h = std::min(tile_h, height - y);
      t.lat_x = x / 16;
      t.lat_y = y / 16;
      ZJAI_TRY(extent(t.img_x, t.img_w, latent_w, &t.lat_w));
      ZJAI_TRY(extent(t.img_y, t.img_h, latent_h, &t.lat_h));
      if (t.lat_x + t.lat_w > latent_w || t.lat_y + t.lat_h > latent_h)
        return fail(ZJAI_INVALID_DATA, "synthesis tile outside the latent");
      const int left = t.img_x == 0 ? 0 : half, top = t.img_y == 0 ? 0 : half;
      const int right = t.img_x + t.img_w >= width ? 0 : half;
      const int bottom = t.img_y + t.img_h >= height ? 0 : half;
      if (t.img_w <= left + right || t.img_h <= top + bottom)
        return fail(ZJAI_INVALID_DATA, "synthesis tile is all overlap");
      t.core_x = t.img_x + left;
      t.core_y = t.img_y + top;
      t.core_w = t.img_w - left - right;
      t.core_h = t.img_h - top - bottom;
      t.off_x = left;
      t.off_y = top;
      out->push_back(t);
    }
  return ZJAI_OK;
}

// Analysis tiling (encoder/tiles.rs:51-156): above ENC_SAMPLES_PER_TILE samples per plane the
// encoder analyses overlapping tiles of floor(sqrt(n)) samples rounded up to the latent grid and
// keeps each tile's latent core (half the overlap trimmed from interior sides).
int analysis_tiles(int ccs, int h, int w, int lh, int lw, std::vector<std::array<int, 14>>* out) {
  static const int kSamples[2] = {1048576, 262144}, kOverlap[2] = {64, 32}, kDown[2] = {16, 8};
  out->clear();
  if (ccs < 0 || ccs > 1 || h <= 0 || w <= 0) return fail(ZJAI_INVALID_ARGUMENT, "analysis tiles");
  if ((long long)kSamples[ccs] >= (long long)h * w) {
    out->push_back({0, 0, w, h, 0, 0, lw, lh, 0, 0, lw, lh, 0, 0});
    return ZJAI_OK;
  }
  const int d = kDown[ccs], overlap = kOverlap[ccs];
  const int size = cdiv((int)std::floor(std::sqrt((double)kSamples[ccs])), d) * d;
  const int tile_h = std::min(size, h), tile_w = std::min(size, w);
  if (tile_h <= overlap || tile_w <= overlap)
    return fail(ZJAI_INVALID_DATA, "analysis tile not larger than overlap");
  const int o = overlap / 2 / d;
  auto latent_len = [&](int pos, int len, int full, int* r) {
    if (len % d && cdiv(pos + len, d) < full)
      return fail(ZJAI_INVALID_DATA, "unaligned analysis tile inside the plane");
    *r = cdiv(len, d);
    return (int)ZJAI_OK;
  };
  for (int y = 0; y < h - overlap; y += tile_h - overlap)
    for (int x = 0; x < w - overlap; x += tile_w - overlap) {
      const int iw = std::min(tile_w, w - x), ih = std::min(tile_h, h - y);
      int lw_t, lh_t;
      ZJAI_TRY(latent_len(x, iw, lw, &lw_t));
      ZJAI_TRY(latent_len(y, ih, lh, &lh_t));
      const int left = x == 0 ? 0 : o, top = y == 0 ? 0 : o;
      const int right = x + iw >= w ? 0 : o, bottom = y + ih >= h ? 0 : o;
      if (lw_t < left + right || lh_t < top + bottom)
        return fail(ZJAI_INVALID_DATA, "analysis tile is all overlap");
      out->push_back({x, y, iw, ih, x / d, y / d, lw_t, lh_t, x / d + left, y / d + top,
                      lw_t - left - right, lh_t - top - bottom, left, top});
    }
  return ZJAI_OK;
}

void synth_out_size(int kind, int op, int h, int w, int* oh, int* ow) {
  int f;
  if (op == ZJAI_HOP)
    f = kind == ZJAI_SYN_Y ? 2 : 4;
  else
    f = kind == ZJAI_SYN_Y ? 4 : 8;
  *oh = f * cdiv(h, f);
  *ow = f * cdiv(w, f);
}

}  // namespace zjai
