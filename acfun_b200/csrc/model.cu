// model.cu — ACFUN0 loader, load-time fuser and the device-resident executor.
//
// Format and fusion rules follow hit-droid/Acfun src/model.cpp:
//   parse   :106-196  magic "ACFUN0", u32 version, inC/inH/inW, num_layers, records
//   fuse    :198-247  Conv/FC/ConvGrouped absorb [ReLU]? then [BN with ch == Cout] (folded
//                     into weight/bias, :69-95); a ReLU followed by MaxPool is dropped
//                     (:220-224, :232 — kept for parity although Pool(ReLU(x)) != Pool(x) for
//                     all-negative windows); MaxPool absorbs a following ReLU (:241)
//   execute :274-349  ping-pong buffers, FC flattens NHWC, Softmax over the whole per-image
//                     tensor (:335), standalone ReLU / BN in place
// Differences by design: records are bounds-checked (a truncated or corrupt file returns
// NULL with error code 5 instead of reading past the blob), weights live on the GPU, and
// acfun_model_infer_batch runs n images through each layer at once (batch-1 semantics per
// image, Softmax per image).
// Format extension (no counterpart in the reference, whose int8 path has no model format):
//   8 ConvInt8  u32 KH, KW, Cout, stride, pad | f32 act_max | f32 wscale[Cout] | f32 b[Cout] |
//               s8 wq[KH*KW*Cin*Cout] | zero bytes to the next multiple of 4
// an already quantised dense convolution (acfun_quantize_weights output of the BN-folded
// weights): it runs through the int8 router like a Conv of an int8-mode model, without
// re-quantising at load.  act_max = 0: one activation scale per image from that image's
// max|x| (the reference's per-call definition, conv_int8.cpp:75-77); act_max > 0: a stored
// calibration range used as every image's max|x| (inputs beyond it saturate).  A ReLU after
// it is fused like a Conv's; a BN after it stays a layer of its own (the stored weights
// cannot absorb it).
#include <algorithm>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <memory>
#include <mutex>
#include <vector>

#include "api_export.cuh"
#include "conv.cuh"
#include "gemm.cuh"
#include "ops.cuh"
#include "runtime.cuh"

namespace acf {

struct MLayer {
  int type = 0;
  int p[8] = {0};
  size_t wn = 0;
  const float* w_host = nullptr;  // into the blob or into `owned`
  const float* b_host = nullptr;
  float* w = nullptr;  // device copies
  float* b = nullptr;
  int act = 0;
  int post_relu = 0;
  int8_t* wq = nullptr;  // int8 mode: per-column quantised conv weights (device)
  float* wqs = nullptr;  // and their scales
  const int8_t* wq_host = nullptr;  // ConvInt8 records: the stored wq / scales (into the blob)
  const float* ws_host = nullptr;
  float act_max = 0.0f;  // ConvInt8: stored activation range (0: measured per image)
  void* wsplit = nullptr;  // bf16 hi / lo split of w for the split-activation conv route
};

}  // namespace acf

struct AcfunModel {
  int inC = 0, inH = 0, inW = 0;
  std::vector<acf::MLayer> layers;
  std::vector<unsigned char> blob;
  std::vector<std::unique_ptr<float[]>> owned;
  int outSize = 0;
  int device = 0;
  float* dparams = nullptr;  // all weights / biases in one device allocation
  float* buf[2] = {nullptr, nullptr};
  size_t bufcap = 0;         // floats per buffer
  std::mutex mu;
  bool int8 = false;         // dense convs through the int8 router, one scale per image
  void* dq = nullptr;        // device allocation of all layers' wq / wqs (int8 mode)
  void* dq8 = nullptr;       // device copies of the ConvInt8 records' wq / wqs
  bool has_int8_layers = false;
};

namespace acf {

static bool rd_u32(const std::vector<unsigned char>& b, size_t& o, unsigned& v) {
  if (o + 4 > b.size()) return false;
  v = (unsigned)b[o] | ((unsigned)b[o + 1] << 8) | ((unsigned)b[o + 2] << 16) |
      ((unsigned)b[o + 3] << 24);
  o += 4;
  return true;
}

static bool rd_f32(const std::vector<unsigned char>& b, size_t& o, size_t n, const float*& p) {
  if (n > (b.size() - o) / 4 || o > b.size()) return false;
  p = reinterpret_cast<const float*>(b.data() + o);
  o += n * 4;
  return true;
}

// model.cpp:69-95, group-aware; host arithmetic without contraction
static void fold_bn(MLayer& F, const MLayer& bn, int Cout, AcfunModel* m) {
  const int ch = bn.p[0];
  const float* mean = bn.w_host;
  const float* var = mean + ch;
  const float* gamma = var + ch;
  const float* beta = gamma + ch;
  const int groups = F.p[5];
  const int Cout_per = groups > 1 ? Cout / groups : Cout;
  const size_t per_in = F.wn / (size_t)Cout;
  std::unique_ptr<float[]> nw(new float[F.wn]), nb(new float[Cout]);
  memcpy(nw.get(), F.w_host, F.wn * 4);
  for (int c = 0; c < Cout; ++c) {
    volatile float scale = gamma[c] / sqrtf(var[c] + 1e-5f);
    volatile float ms = mean[c] * scale;
    const float shift = beta[c] - ms;
    const int gc = groups > 1 ? c / Cout_per : 0, oc = groups > 1 ? c % Cout_per : c;
    for (size_t t = 0; t < per_in; ++t) nw[(size_t)gc * Cout_per * per_in + t * Cout_per + oc] *= scale;
    volatile float bs = (F.b_host ? F.b_host[c] : 0.0f) * scale;
    nb[c] = bs + shift;
  }
  F.w_host = nw.get();
  F.b_host = nb.get();
  m->owned.push_back(std::move(nw));
  m->owned.push_back(std::move(nb));
}

static AcfunModel* load_blob(std::vector<unsigned char>&& blob) {
  std::unique_ptr<AcfunModel> m(new AcfunModel());
  m->blob = std::move(blob);
  const auto& b = m->blob;
  if (b.size() < 6 + 16 || memcmp(b.data(), "ACFUN0", 6) != 0) {
    set_error(kFormat, "acfun_model_load: bad magic or short file");
    return nullptr;
  }
  size_t o = 10;
  unsigned inC, inH, inW, num;
  rd_u32(b, o, inC);
  rd_u32(b, o, inH);
  rd_u32(b, o, inW);
  rd_u32(b, o, num);
  if (inC == 0 || inH == 0 || inW == 0 || inC > 65536 || inH > 65536 || inW > 65536) {
    set_error(kFormat, "acfun_model_load: bad input dims %u x %u x %u", inC, inH, inW);
    return nullptr;
  }
  m->inC = (int)inC;
  m->inH = (int)inH;
  m->inW = (int)inW;
  std::vector<MLayer> raw;
  raw.reserve(num < 100000 ? num : 100000);
  int prevC = (int)inC;
  auto bad = [&](unsigned i) {
    set_error(kFormat, "acfun_model_load: layer %u truncated or malformed", i);
    return (AcfunModel*)nullptr;
  };
  for (unsigned i = 0; i < num; ++i) {
    MLayer L;
    unsigned t;
    if (!rd_u32(b, o, t)) return bad(i);
    L.type = (int)t;
    switch (t) {
      case 1:
      case 7: {
        unsigned v[6] = {0, 0, 0, 0, 0, 1};
        for (int k = 0; k < (t == 7 ? 6 : 5); ++k)
          if (!rd_u32(b, o, v[k])) return bad(i);
        if (!v[0] || !v[1] || !v[2] || !v[3] || !v[5] || v[0] > 64 || v[1] > 64 ||
            v[2] > (1u << 20) || (t == 7 && (prevC % v[5] || v[2] % v[5])))
          return bad(i);
        for (int k = 0; k < 6; ++k) L.p[k] = (int)v[k];
        if (t == 1) L.p[5] = 0;
        L.wn = (size_t)v[0] * v[1] * prevC * v[2] / (t == 7 ? v[5] : 1);
        if (!rd_f32(b, o, L.wn, L.w_host) || !rd_f32(b, o, v[2], L.b_host)) return bad(i);
        L.p[6] = prevC;
        prevC = (int)v[2];
        break;
      }
      case 8: {
        unsigned v[5];
        for (int k = 0; k < 5; ++k)
          if (!rd_u32(b, o, v[k])) return bad(i);
        if (!v[0] || !v[1] || !v[2] || !v[3] || v[0] > 64 || v[1] > 64 || v[2] > (1u << 20))
          return bad(i);
        for (int k = 0; k < 5; ++k) L.p[k] = (int)v[k];
        L.p[5] = 0;
        const float* am = nullptr;
        if (!rd_f32(b, o, 1, am) || !(am[0] >= 0.0f) || !(am[0] < 3.0e38f)) return bad(i);
        L.act_max = am[0];
        L.wn = (size_t)v[0] * v[1] * prevC * v[2];
        if (!rd_f32(b, o, v[2], L.ws_host) || !rd_f32(b, o, v[2], L.b_host)) return bad(i);
        const size_t padded = (L.wn + 3) / 4 * 4;
        if (o > b.size() || padded > b.size() - o) return bad(i);
        L.wq_host = reinterpret_cast<const int8_t*>(b.data() + o);
        o += padded;
        L.p[6] = prevC;
        prevC = (int)v[2];
        m->has_int8_layers = true;
        break;
      }
      case 2: {
        unsigned Cout, inDim;
        if (!rd_u32(b, o, Cout) || !rd_u32(b, o, inDim) || !Cout || !inDim) return bad(i);
        L.p[0] = (int)Cout;
        L.p[1] = (int)inDim;
        L.wn = (size_t)inDim * Cout;
        if (!rd_f32(b, o, L.wn, L.w_host) || !rd_f32(b, o, Cout, L.b_host)) return bad(i);
        prevC = (int)Cout;
        break;
      }
      case 3:
      case 5:
        break;
      case 4: {
        unsigned v[3];
        for (int k = 0; k < 3; ++k)
          if (!rd_u32(b, o, v[k])) return bad(i);
        if (!v[0] || !v[1]) return bad(i);
        L.p[0] = (int)v[0];
        L.p[1] = (int)v[1];
        L.p[2] = (int)v[2];
        break;
      }
      case 6: {
        unsigned ch;
        if (!rd_u32(b, o, ch) || !ch) return bad(i);
        L.p[0] = (int)ch;
        L.wn = (size_t)ch * 4;
        if (!rd_f32(b, o, L.wn, L.w_host)) return bad(i);
        break;
      }
      default:
        set_error(kFormat, "acfun_model_load: unknown layer type %u at layer %u", t, i);
        return nullptr;
    }
    raw.push_back(L);
  }
  // ---- fusion (model.cpp:198-247).  ACFUN_PARITY_STRICT=0 corrects the reference's two
  // order quirks instead of reproducing them: a ReLU right before a MaxPool is kept, and
  // Conv -> ReLU -> BN keeps the BN as its own layer after the activation (the reference
  // folds it into the conv, i.e. applies BN before ReLU).
  const char* strict_env = getenv("ACFUN_PARITY_STRICT");
  const bool strict = !(strict_env && strict_env[0] == '0' && strict_env[1] == 0);
  const int n = (int)raw.size();
  std::vector<char> consumed(n, 0);
  for (int i = 0; i < n; ++i) {
    if (consumed[i]) continue;
    MLayer& L = raw[i];
    if (L.type == 1 || L.type == 2 || L.type == 7 || L.type == 8) {
      MLayer F = L;
      F.act = 0;
      const int Cout = L.type == 2 ? L.p[0] : L.p[2];
      int j = i + 1, relu_idx = -1;
      if (j < n && raw[j].type == 3) relu_idx = j++;
      if (L.type != 8 && j < n && raw[j].type == 6 && raw[j].p[0] == Cout &&
          (strict || relu_idx < 0)) {
        fold_bn(F, raw[j], Cout, m.get());
        consumed[j] = 1;
      }
      if (relu_idx >= 0) {
        consumed[relu_idx] = 1;
        F.act = (strict && j < n && raw[j].type == 4) ? 0 : 1;
      }
      m->layers.push_back(F);
    } else if (L.type == 3) {
      if (strict && i + 1 < n && raw[i + 1].type == 4) {
        consumed[i] = 1;
        continue;
      }
      m->layers.push_back(L);
    } else if (L.type == 4) {
      MLayer F = L;
      if (i + 1 < n && raw[i + 1].type == 3) {
        F.post_relu = 1;
        consumed[i + 1] = 1;
      }
      m->layers.push_back(F);
    } else {
      m->layers.push_back(L);
    }
  }
  // ---- shape check and device upload
  int H = m->inH, W = m->inW, C = m->inC;
  size_t total = 0, maxact = (size_t)H * W * C;
  for (auto& L : m->layers) {
    if (L.type == 1 || L.type == 7 || L.type == 8) {
      if (L.p[6] != C) {
        set_error(kFormat, "acfun_model_load: channel mismatch");
        return nullptr;
      }
      const int OH = (H + 2 * L.p[4] - L.p[0]) / L.p[3] + 1, OW = (W + 2 * L.p[4] - L.p[1]) / L.p[3] + 1;
      if (OH <= 0 || OW <= 0) {
        set_error(kFormat, "acfun_model_load: conv produces an empty map");
        return nullptr;
      }
      H = OH;
      W = OW;
      C = L.p[2];
      total += (L.type == 8 ? 0 : L.wn) + (size_t)C;  // ConvInt8 weights live in dq8
    } else if (L.type == 2) {
      if ((size_t)L.p[1] != (size_t)H * W * C) {
        set_error(kFormat, "acfun_model_load: FC inDim %d != %d", L.p[1], H * W * C);
        return nullptr;
      }
      H = W = 1;
      C = L.p[0];
      total += L.wn + (size_t)C;
    } else if (L.type == 4) {
      const int OH = (H + 2 * L.p[2] - L.p[0]) / L.p[1] + 1, OW = (W + 2 * L.p[2] - L.p[0]) / L.p[1] + 1;
      if (OH <= 0 || OW <= 0) {
        set_error(kFormat, "acfun_model_load: pool produces an empty map");
        return nullptr;
      }
      H = OH;
      W = OW;
    } else if (L.type == 6) {
      total += L.wn;
    }
    const size_t a = (size_t)H * W * C;
    if (a > maxact) maxact = a;
  }
  m->outSize = H * W * C;
  m->bufcap = 0;
  m->device = current_device();
  DeviceState* ds = device_state();
  if (!ds || !ACF_CUDA_OK(cudaSetDevice(m->device))) return nullptr;
  if (!ACF_CUDA_OK(cudaMalloc(&m->dparams, (total ? total : 1) * 4))) return nullptr;
  size_t off = 0;
  for (auto& L : m->layers) {
    if (L.wn && L.type != 8) {
      L.w = m->dparams + off;
      if (!ACF_CUDA_OK(cudaMemcpy(L.w, L.w_host, L.wn * 4, cudaMemcpyHostToDevice))) return nullptr;
      off += L.wn;
    }
    if (L.type == 1 || L.type == 7 || L.type == 2 || L.type == 8) {
      const int Cout = L.type == 2 ? L.p[0] : L.p[2];
      L.b = m->dparams + off;
      if (!ACF_CUDA_OK(cudaMemcpy(L.b, L.b_host, (size_t)Cout * 4, cudaMemcpyHostToDevice)))
        return nullptr;
      off += Cout;
    }
  }
  // ConvInt8 records: wq and scales, each in a 16-byte aligned slot of one allocation
  if (m->has_int8_layers) {
    size_t q = 0;
    for (auto& L : m->layers)
      if (L.type == 8) q += align_up(L.wn, 16) + align_up((size_t)L.p[2] * 4, 16);
    if (!ACF_CUDA_OK(cudaMalloc(&m->dq8, q))) return nullptr;
    unsigned char* base = static_cast<unsigned char*>(m->dq8);
    for (auto& L : m->layers) {
      if (L.type != 8) continue;
      const size_t cb = (size_t)L.p[2] * 4;
      L.wq = reinterpret_cast<int8_t*>(base);
      L.wqs = reinterpret_cast<float*>(base + align_up(L.wn, 16));
      if (!ACF_CUDA_OK(cudaMemcpy(L.wq, L.wq_host, L.wn, cudaMemcpyHostToDevice)) ||
          !ACF_CUDA_OK(cudaMemcpy(L.wqs, L.ws_host, cb, cudaMemcpyHostToDevice)))
        return nullptr;
      base += align_up(L.wn, 16) + align_up(cb, 16);
    }
  }
  (void)maxact;
  return m.release();
}

static size_t max_activation(const AcfunModel* m) {
  int H = m->inH, W = m->inW, C = m->inC;
  size_t mx = (size_t)H * W * C;
  for (auto& L : m->layers) {
    if (L.type == 1 || L.type == 7 || L.type == 8) {
      H = (H + 2 * L.p[4] - L.p[0]) / L.p[3] + 1;
      W = (W + 2 * L.p[4] - L.p[1]) / L.p[3] + 1;
      C = L.p[2];
    } else if (L.type == 2) {
      H = W = 1;
      C = L.p[0];
    } else if (L.type == 4) {
      H = (H + 2 * L.p[2] - L.p[0]) / L.p[1] + 1;
      W = (W + 2 * L.p[2] - L.p[0]) / L.p[1] + 1;
    }
    size_t a = (size_t)H * W * C;
    // room for the zero-padded split form when a convolution reads this output
    const size_t li = (size_t)(&L - m->layers.data());
    if (li + 1 < m->layers.size() && m->layers[li + 1].type == 1) {
      const int p = m->layers[li + 1].p[4];
      a = std::max(a, (size_t)(H + 2 * p) * (W + 2 * p) * C);
    }
    if (a > mx) mx = a;
  }
  return mx;
}

// Runs `n` images (batch-1 semantics each) from device input `x` into device output `y`.
static bool run_model(Call& c, AcfunModel* m, int n, const float* x, float* y) {
  const size_t need = max_activation(m) * (size_t)n;
  if (need > m->bufcap) {
    cudaStreamSynchronize(c.stream());
    cudaFree(m->buf[0]);
    cudaFree(m->buf[1]);
    m->buf[0] = m->buf[1] = nullptr;
    m->bufcap = 0;
    if (!ACF_CUDA_OK(cudaMalloc(&m->buf[0], need * 4)) ||
        !ACF_CUDA_OK(cudaMalloc(&m->buf[1], need * 4))) {
      c.fail();
      return false;
    }
    m->bufcap = need;
  }
  int H = m->inH, W = m->inW, C = m->inC;
  const float* cur = x;
  int which = 0;
  const size_t nl = m->layers.size();
  // The current activation may be held in split form (cs): the zero-padded bf16 hi / lo planes
  // the next convolution's 3xBF16 implicit GEMM reads, written directly by the layer that
  // produced it.  Only a layer whose consumer is such a convolution produces it.
  SplitAct cs;
  bool in_split = false;
  auto split_target = [&](size_t j, int Hn, int Wn, int Cn, float* buf, SplitAct& os) -> bool {
    if (m->int8 || j >= nl || m->layers[j].type != 1) return false;
    const auto& Nx = m->layers[j];
    if (!conv_split_ok(Hn, Wn, Cn, Nx.p[0], Nx.p[1], Nx.p[2], Nx.p[3], Nx.p[4])) return false;
    os.base = buf;
    os.N = n;
    os.H = Hn;
    os.W = Wn;
    os.C = Cn;
    os.pad = Nx.p[4];
    os.plane = (long long)n * (Hn + 2 * os.pad) * (Wn + 2 * os.pad) * Cn;
    return true;
  };
  // int8 mode: a conv whose output feeds a dense int8 conv directly accumulates that output's
  // per-image max |y| (the next conv's activation scale) in its epilogue as it stores it, so
  // the next conv skips its absmax pass; cur_max is the maximum of `cur` when its producer did
  // so.  (A max-pool producer does not: per-image reductions in its grid-stride order cost
  // more than the absmax pass they save.)
  unsigned* imax[2] = {nullptr, nullptr};
  unsigned* smax = nullptr;  // a ConvInt8 layer's stored activation range, per image
  const unsigned* cur_max = nullptr;
  int mwhich = 0;
  if (m->int8 || m->has_int8_layers) {
    imax[0] = static_cast<unsigned*>(c.scratch((size_t)n * 4));
    imax[1] = static_cast<unsigned*>(c.scratch((size_t)n * 4));
    smax = static_cast<unsigned*>(c.scratch((size_t)n * 4));
    if (!imax[0] || !imax[1] || !smax) return false;
  }
  auto int8_layer = [&](const MLayer& Lj) {  // this layer runs through the int8 router
    return Lj.wq && ((m->int8 && Lj.type == 1) || Lj.type == 8);
  };
  auto pool2_follows = [&](size_t j) -> bool {  // layer j + 1 is MaxPool(2, 2, 0)
    if (j + 1 >= nl || m->layers[j + 1].type != 4) return false;
    const auto& P = m->layers[j + 1];
    return P.p[0] == 2 && P.p[1] == 2 && P.p[2] == 0;
  };
  auto max_for = [&](size_t j) -> unsigned* {
    // (a consumer with a stored activation range needs no measured maximum)
    if (j >= nl || !int8_layer(m->layers[j]) || m->layers[j].act_max > 0.0f) return nullptr;
    unsigned* d = imax[mwhich];
    mwhich ^= 1;
    return ACF_CUDA_OK(cudaMemsetAsync(d, 0, (size_t)n * 4, c.stream())) ? d : nullptr;
  };
  for (size_t li = 0; li < nl; ++li) {
    auto& L = m->layers[li];
    float* next = m->buf[which];
    bool ok = true;
    const unsigned* in_max = cur_max;
    cur_max = nullptr;
    // A standalone ReLU right after a Conv / FC (the loader keeps Conv->BN->ReLU's ReLU
    // separate, model.cpp:211-226) is applied in that layer's epilogue instead of a pass.
    int act = L.act;
    if ((L.type == 1 || L.type == 2 || L.type == 7 || L.type == 8) && li + 1 < nl &&
        m->layers[li + 1].type == 3) {
      act = 1;
      ++li;
    }
    switch (L.type) {
      case 1:
      case 7:
      case 8: {
        const int KH = L.p[0], KW = L.p[1], Cout = L.p[2], st = L.p[3], pd = L.p[4];
        const int groups = L.type == 7 ? L.p[5] : 1;
        if (int8_layer(L)) {
          if (L.act_max > 0.0f) {
            // a stored activation range: every image's max|x| is that constant
            unsigned bits;
            memcpy(&bits, &L.act_max, 4);
            ok = fill_u32_dev(c, smax, bits, n);
            in_max = smax;
          }
          // int8 mode: acfun_conv2d_int8 per image (the reference's int8 model harness); a
          // small-K conv followed by MaxPool(2, 2, 0) runs fused
          // (one max_for per layer: a second call would hand out the array in_max points at)
          const bool pool_next = li + 1 < nl && m->layers[li + 1].type == 4;
          unsigned* om_pool = pool_next ? max_for(li + 2) : nullptr;  // the pool's consumer
          if (pool_next) {
            const auto& P = m->layers[li + 1];
            bool fused = false;
            ok = ok && conv_int8_pool_dev(c, cur, n, H, W, C, L.wq, L.wqs, L.b, KH, KW, Cout, st, pd,
                                          act, P.p[0], P.p[1], P.p[2], P.post_relu, next, &fused,
                                          om_pool, L.act_max > 0.0f ? smax : nullptr);
            if (ok && fused) cur_max = om_pool;
            if (ok && fused) {
              H = (H + 2 * pd - KH) / st + 1;
              W = (W + 2 * pd - KW) / st + 1;
              H = (H + 2 * P.p[2] - P.p[0]) / P.p[1] + 1;
              W = (W + 2 * P.p[2] - P.p[0]) / P.p[1] + 1;
              C = Cout;
              cur = next;
              which ^= 1;
              ++li;
              break;
            }
          }
          // a following MaxPool(2, 2, 0) runs in the GEMM epilogue when the route allows
          const bool pooled = pool2_follows(li) && int8_pool_ok(H, W, C, KH, KW, Cout, st, pd);
          unsigned* om = pooled ? om_pool : (ok && !pool_next ? max_for(li + 1) : nullptr);
          ok = ok && conv2d_int8_batch_dev(c, cur, n, H, W, C, L.wq, L.wqs, L.b, KH, KW, Cout, st,
                                           pd, next, pooled ? (act | m->layers[li + 1].post_relu) : act,
                                           in_max, om, pooled);
          cur_max = om;
          H = (H + 2 * pd - KH) / st + 1;
          W = (W + 2 * pd - KW) / st + 1;
          if (pooled) {
            H /= 2;
            W /= 2;
            ++li;
          }
          C = Cout;
          cur = next;
          which ^= 1;
          break;
        }
        const int OHc = (H + 2 * pd - KH) / st + 1, OWc = (W + 2 * pd - KW) / st + 1;
        // Conv -> MaxPool: the pooled output straight from the conv when the pair fuses
        // (written in split form when the layer after the pool is a split convolution)
        if (!in_split && groups == 1 && li + 1 < nl && m->layers[li + 1].type == 4) {
          const auto& P = m->layers[li + 1];
          const int PH = (OHc + 2 * P.p[2] - P.p[0]) / P.p[1] + 1;
          const int PW = (OWc + 2 * P.p[2] - P.p[0]) / P.p[1] + 1;
          SplitAct os;
          bool fused = false, as_split = false;
          if (split_target(li + 2, PH, PW, Cout, next, os)) {
            ok = split_border_dev(c, os) &&
                 conv_pool_dev(c, cur, n, H, W, C, L.w, L.b, KH, KW, Cout, st, pd, act, P.p[0],
                               P.p[1], P.p[2], P.post_relu, next, &fused, &os);
            as_split = fused;
          }
          if (ok && !fused)
            ok = conv_pool_dev(c, cur, n, H, W, C, L.w, L.b, KH, KW, Cout, st, pd, act, P.p[0],
                               P.p[1], P.p[2], P.post_relu, next, &fused);
          if (ok && fused) {
            H = PH;
            W = PW;
            C = Cout;
            cur = next;
            which ^= 1;
            in_split = as_split;
            if (as_split) cs = os;
            ++li;
            break;
          }
        }
        // 3xBF16 implicit GEMM from / to split activations, weights split once per model
        if (ok && groups == 1 && (in_split || conv_split_ok(H, W, C, KH, KW, Cout, st, pd))) {
          if (!L.wsplit) {
            if (!ACF_CUDA_OK(cudaMalloc(&L.wsplit, (size_t)split_weight_bytes(KH * KW, C, Cout))) ||
                !split_weights_dev(c, L.w, KH * KW, C, Cout, L.wsplit)) {
              c.fail();
              return false;
            }
          }
          // a following MaxPool(2, 2, 0) runs in the conv's epilogue (row-pair tiles)
          const bool pooled = pool2_follows(li) && st == 1 && (H + 2 * pd) % 2 == 0 && OHc >= 2 &&
                              OWc >= 2;
          const int oh = pooled ? OHc / 2 : OHc, ow = pooled ? OWc / 2 : OWc;
          SplitAct os;
          const bool want = split_target(li + (pooled ? 2 : 1), oh, ow, Cout, next, os);
          if (want) ok = split_border_dev(c, os);
          ok = ok && conv_tc_split_dev(c, in_split ? nullptr : cur, in_split ? &cs : nullptr, n, H, W,
                                       C, L.w, L.wsplit, L.b, KH, KW, Cout, pd, next,
                                       want ? &os : nullptr,
                                       pooled ? (act | m->layers[li + 1].post_relu) : act, pooled);
          if (pooled) ++li;
          H = oh;
          W = ow;
          C = Cout;
          cur = next;
          which ^= 1;
          in_split = want;
          if (want) cs = os;
          break;
        }
        ok = ok && conv2d_dev(c, cur, n, H, W, C, L.w, L.b, KH, KW, Cout, st, pd, groups, next, act);
        H = (H + 2 * pd - KH) / st + 1;
        W = (W + 2 * pd - KW) / st + 1;
        C = Cout;
        cur = next;
        which ^= 1;
        break;
      }
      case 2: {
        const int Cout = L.p[0], inDim = H * W * C;
        // the weights' 3xBF16 split is made once and cached with the layer
        Operand bs;
        const Operand* bsp = nullptr;
        if (fp32_math(Fp32Use::Conv) == Fp32Math::BF16X3) {
          if (!L.wsplit) {
            if (!ACF_CUDA_OK(cudaMalloc(&L.wsplit, (size_t)bf16x2_bytes(inDim, Cout)))) {
              c.fail();
              return false;
            }
            to_bf16x2(c, L.w, inDim, Cout, Cout, L.wsplit);
          }
          bs.p = L.wsplit;
          bs.ld = (long long)align_up((size_t)Cout, 8);
          bs.op_stride = (long long)inDim * bs.ld;
          bsp = &bs;
        }
        ok = c.ok() && gemm_f32(c, cur, inDim, L.w, Cout, n, Cout, inDim, next, Cout, L.b, act,
                                Fp32Use::Conv, bsp);
        H = W = 1;
        C = Cout;
        cur = next;
        which ^= 1;
        break;
      }
      case 3:
        if (cur == x) {  // never write the caller's input: ReLU out of place
          ok = ACF_CUDA_OK(cudaMemcpyAsync(next, cur, (size_t)n * H * W * C * 4,
                                           cudaMemcpyDeviceToDevice, c.stream()));
          cur = next;
          which ^= 1;
        }
        ok = ok && relu_dev(c, const_cast<float*>(cur), (long long)n * H * W * C, 0);
        break;
      case 4: {
        const int pool = L.p[0], st = L.p[1], pd = L.p[2];
        const int PH = (H + 2 * pd - pool) / st + 1, PW = (W + 2 * pd - pool) / st + 1;
        SplitAct os;
        const bool want = C % 16 == 0 && split_target(li + 1, PH, PW, C, next, os);
        if (want) ok = split_border_dev(c, os);
        ok = ok && maxpool_dev(c, cur, n, H, W, C, pool, st, pd, next, L.post_relu,
                               want ? &os : nullptr);
        H = PH;
        W = PW;
        cur = next;
        which ^= 1;
        in_split = want;
        if (want) cs = os;
        break;
      }
      case 5:
        ok = softmax_dev(c, cur, n, H * W * C, next);
        cur = next;
        which ^= 1;
        break;
      case 6: {
        if (cur == x) {
          ok = ACF_CUDA_OK(cudaMemcpyAsync(next, cur, (size_t)n * H * W * C * 4,
                                           cudaMemcpyDeviceToDevice, c.stream()));
          cur = next;
          which ^= 1;
        }
        const int ch = L.p[0];
        const size_t per = (size_t)H * W * C;
        // per image: the reference's `spatial = size / channels` floor is per call
        if (per % ch == 0) {
          ok = ok && batchnorm_dev(c, const_cast<float*>(cur), (int)(per * n), ch, L.w, L.w + ch,
                                   L.w + 2 * ch, L.w + 3 * ch, 1e-5f);
        } else {
          for (int k = 0; k < n && ok; ++k)
            ok = batchnorm_dev(c, const_cast<float*>(cur) + per * k, (int)per, ch, L.w, L.w + ch,
                               L.w + 2 * ch, L.w + 3 * ch, 1e-5f);
        }
        break;
      }
    }
    if (!ok) {
      c.fail();
      return false;
    }
  }
  return ACF_CUDA_OK(cudaMemcpyAsync(y, cur, (size_t)n * m->outSize * 4, cudaMemcpyDeviceToDevice,
                                     c.stream()));
}

}  // namespace acf

using namespace acf;

extern "C" AcfunModel* acfun_model_load(const char* path) {
  if (!path) return nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) {
    set_error(kInvalid, "acfun_model_load: cannot open %s", path);
    return nullptr;
  }
  std::vector<unsigned char> blob;
  fseek(f, 0, SEEK_END);
  const long sz = ftell(f);
  fseek(f, 0, SEEK_SET);
  if (sz > 0) {
    blob.resize((size_t)sz);
    if (fread(blob.data(), 1, (size_t)sz, f) != (size_t)sz) {
      fclose(f);
      set_error(kFormat, "acfun_model_load: short read");
      return nullptr;
    }
  }
  fclose(f);
  return load_blob(std::move(blob));
}

extern "C" void acfun_model_destroy(AcfunModel* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  cudaDeviceSynchronize();
  cudaFree(m->dparams);
  cudaFree(m->dq);
  cudaFree(m->dq8);
  for (auto& L : m->layers) cudaFree(L.wsplit);
  cudaFree(m->buf[0]);
  cudaFree(m->buf[1]);
  delete m;
}

extern "C" int acfun_model_output_size(AcfunModel* m) { return m ? m->outSize : 0; }

extern "C" void acfun_model_input_dims(AcfunModel* m, int* Cin, int* Hin, int* Win) {
  if (!m) return;
  if (Cin) *Cin = m->inC;
  if (Hin) *Hin = m->inH;
  if (Win) *Win = m->inW;
}

extern "C" int acfun_model_infer_batch(AcfunModel* m, int n, const float* input, float* output) {
  if (!m || n <= 0 || !input || !output) return 0;
  std::lock_guard<std::mutex> g(m->mu);
  tctx().device = m->device;
  Call c("acfun_model_infer");
  if (!c.ok()) return 0;
  const size_t in_elems = (size_t)n * m->inH * m->inW * m->inC;
  const float* dx = (const float*)c.in(input, in_elems * 4);
  float* dy = (float*)c.out(output, (size_t)n * m->outSize * 4);
  if (!c.ok()) return 0;
  if (!run_model(c, m, n, dx, dy)) {
    c.finish();
    return 0;
  }
  return c.finish() ? m->outSize : 0;
}

// Extension (no counterpart in the reference, whose int8 path has no model format): run every
// dense convolution of the model through the int8 router with one activation scale per image
// -- what the reference's per-image harness does with acfun_quantize_weights +
// acfun_conv2d_int8 -- while FC, pooling, BN and softmax stay fp32.  Weights are quantised
// here, on the host, from the folded fp32 weights.
extern "C" int acfun_model_set_int8(AcfunModel* m, int enable) {
  if (!m) {
    set_error(kInvalid, "acfun_model_set_int8: NULL model");
    return kInvalid;
  }
  std::lock_guard<std::mutex> g(m->mu);
  if (!enable) {
    m->int8 = false;
    return 0;
  }
  if (m->dq) {
    m->int8 = true;
    return 0;
  }
  // sizes: per dense conv K*Cout bytes of wq + Cout floats of scales (16-byte aligned slots)
  size_t total = 0;
  for (auto& L : m->layers) {
    if (L.type != 1) continue;
    const size_t cout = (size_t)L.p[2];
    total += align_up(L.wn, 16) + align_up(cout * 4, 16);
  }
  std::vector<unsigned char> host(total);
  size_t off = 0;
  std::vector<size_t> offs;
  for (auto& L : m->layers) {
    if (L.type != 1) continue;
    const int cout = L.p[2];
    const int K = (int)(L.wn / (size_t)cout);
    int8_t* q = reinterpret_cast<int8_t*>(host.data() + off);
    float* sc = reinterpret_cast<float*>(host.data() + off + align_up(L.wn, 16));
    acfun_quantize_weights(L.w_host, K, cout, sc, q);
    offs.push_back(off);
    off += align_up(L.wn, 16) + align_up((size_t)cout * 4, 16);
  }
  tctx().device = m->device;
  if (!ACF_CUDA_OK(cudaSetDevice(m->device))) return kCuda;
  void* d = nullptr;
  if (total && (!ACF_CUDA_OK(cudaMalloc(&d, total)) ||
                !ACF_CUDA_OK(cudaMemcpy(d, host.data(), total, cudaMemcpyHostToDevice)))) {
    cudaFree(d);
    return kCuda;
  }
  size_t k = 0;
  for (auto& L : m->layers) {
    if (L.type != 1) continue;
    unsigned char* base = static_cast<unsigned char*>(d) + offs[k++];
    L.wq = reinterpret_cast<int8_t*>(base);
    L.wqs = reinterpret_cast<float*>(base + align_up(L.wn, 16));
  }
  m->dq = d;
  m->int8 = true;
  return 0;
}

extern "C" int acfun_model_infer(AcfunModel* m, const float* input, float* output) {
  return acfun_model_infer_batch(m, 1, input, output);
}
