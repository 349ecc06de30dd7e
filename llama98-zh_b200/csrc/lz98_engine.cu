// Host side of the B200-native MTP speculative-decoding step: model.bin
// ("L98Z" v5) reader and HBM upload, the device run state (KDA state
// ring, conv ring, MTP KV cache, draft chain), the forward orchestration
// (body verify forward, MTP draft step, MTP prefill/catch-up) and the C ABI
// declared in include/lz98_gpu.h.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>   // types only: the functions are bound at run time (nccl_api)
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <chrono>
#include <initializer_list>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/lz98_gpu.h"
#include "lz98_kernels.cuh"
#include "lz98_sample.cuh"
#include "lz98_umma.cuh"
#include "lz98_rope_table.h"
#include "lz98_ep.cuh"

using namespace lz98;

namespace {

void set_err(char* buf, int len, const char* fmt, const char* a = "") {
  if (buf && len > 0) snprintf(buf, (size_t)len, fmt, a);
}


#define CK(call)                                                              \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess) {                                                  \
      fprintf(stderr, "lz98: CUDA error %s at %s:%d\n", cudaGetErrorString(e_), \
              __FILE__, __LINE__);                                            \
      return LZ98_ERR_CUDA;                                                   \
    }                                                                         \
  } while (0)

struct QW {                       // Q8_0 weight resident in HBM
  int out = 0, in = 0, gs = 0;
  int8_t* q = nullptr;
  float* s = nullptr;
};

struct HQ {                       // host copy while reading
  int out = 0, in = 0, gs = 0;
  std::vector<int8_t> q;
  std::vector<float> s;
};

struct Cfg {
  int vocab, d, nl, seq_len, nh, nkv, hd, inter, nk, nv, kd, vd, conv_k;
  float eps, theta, prf;
  int q_dim, qg_dim, kv_dim, key_dim, val_dim, conv_dim, rot;
  int rank, has_lb;
  float lb;
  int ne, topk, n_shared, moe_ffn, latent, fkdr, renorm, sigm, lat_norm, shared_w, mtp_layers, mtp_ffn;
};

struct DLayer {
  float *in_ln, *post_ln, *conv_w, *a_log, *dt_bias, *o_norm, *router_bias;
  QW inproj, fb, o, moein, up, sh_down;
  int8_t *w13q, *w2q;
  float *w13s, *w2s;
  int w13_gs, w2_gs;
};

struct DMtp {
  float *in_ln, *post_ln, *q_norm, *k_norm, *norm, *pre_h, *pre_e;
  QW fc, qkv, o, gu, down;
};

}  // namespace

struct LZModel {
  Cfg c;
  QW embed;
  float* final_norm = nullptr;
  std::vector<DLayer> L;
  DMtp mtp;
  int dev = 0;                    // the CUDA device the tensors live on
  size_t wbytes = 0;
  std::vector<void*> allocs;
  // column offsets inside the fused projection groups
  int off_q, off_k, off_v, off_g, off_fa, off_b, n_in;
  int off_router, off_down, off_shg, off_shu, n_moe;
  int off_mq, off_mk, off_mv, n_qkv;
};

namespace {

// IEEE binary16 to binary32, exact (every half is a float): sign, then
// zero / subnormal (normalised into a float exponent) / normal / inf-NaN.
float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu, u;
  if (e == 0) {
    if (m == 0) {
      u = sign;
    } else {
      int sh = 0;
      while (!(m & 0x400u)) { m <<= 1; sh++; }
      u = sign | ((uint32_t)(127 - 14 - sh) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 0x1Fu) {
    u = sign | 0x7F800000u | (m << 13);
  } else {
    u = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

struct Reader {
  FILE* f = nullptr;
  bool bad = false;
  int layout = 0;   // Q8_0 scale planes (src/model.c:3510-3556): 0 f32, 1 binary16, 2 binary16 row base + u8
  // one scale plane of ng groups over `rows` rows, decoded to f32
  void scales(float* dst, uint32_t ng, int rows) {
    if (layout == 0) {
      bytes(dst, (size_t)ng * 4);
      return;
    }
    if (layout == 1) {
      std::vector<uint16_t> h(ng);
      bytes(h.data(), (size_t)ng * 2);
      for (uint32_t i = 0; i < ng && !bad; i++) dst[i] = half_to_float(h[i]);
      return;
    }
    if (rows <= 0 || ng % (uint32_t)rows) { bad = true; return; }
    std::vector<uint16_t> hb(rows);
    std::vector<uint8_t> code(ng);
    bytes(hb.data(), (size_t)rows * 2);
    bytes(code.data(), ng);
    const uint32_t gpr = ng / (uint32_t)rows;
    for (uint32_t i = 0; i < ng && !bad; i++) {
      // base * (code / 255), the quotient and the product each rounded to
      // float (the reference's lz_scale_u8_decode)
      volatile float q = (float)code[i] / 255.0f;
      volatile float p = half_to_float(hb[i / gpr]) * q;
      dst[i] = p;
    }
  }
  void bytes(void* p, size_t n) {
    if (!bad && fread(p, 1, n, f) != n) bad = true;
  }
  int i32() { int32_t v = 0; bytes(&v, 4); return v; }
  float f32() { float v = 0; bytes(&v, 4); return v; }
  std::vector<float> ften(size_t n) {
    uint8_t dt = 0; uint32_t cnt = 0;
    bytes(&dt, 1); bytes(&cnt, 4);
    std::vector<float> v;
    if (bad || dt != 0 || cnt != n) { bad = true; return v; }
    v.resize(n);
    bytes(v.data(), n * 4);
    return v;
  }
  HQ qten(int out, int in) {
    HQ t;
    uint8_t dt = 0; uint32_t cnt = 0, gs = 0;
    bytes(&dt, 1); bytes(&cnt, 4); bytes(&gs, 4);
    if (bad || dt != 1 || (long long)cnt != (long long)out * in || gs == 0 || cnt % gs || gs % 32 ||
        in % gs) {
      bad = true;
      return t;
    }
    t.out = out; t.in = in; t.gs = (int)gs;
    t.q.resize(cnt);
    t.s.resize(cnt / gs);
    bytes(t.q.data(), cnt);
    scales(t.s.data(), cnt / gs, out);
    return t;
  }
};

template <typename T>
T* dev_upload(LZModel* m, const T* src, size_t n) {
  T* p = nullptr;
  if (cudaMalloc(&p, n * sizeof(T) + 16) != cudaSuccess) return nullptr;
  cudaMemcpy(p, src, n * sizeof(T), cudaMemcpyHostToDevice);
  m->allocs.push_back(p);
  m->wbytes += n * sizeof(T);
  return p;
}

float* up_f(LZModel* m, const std::vector<float>& v) { return dev_upload(m, v.data(), v.size()); }

// Concatenate tensors of equal in-dim and group size along the output
// dimension into one fused weight (rows stay whole, so every output row's
// arithmetic is exactly that of its own tensor).
bool up_group(LZModel* m, const std::vector<const HQ*>& parts, QW* out) {
  int in = parts[0]->in, gs = parts[0]->gs, rows = 0;
  for (auto* p : parts) {
    if (p->in != in || p->gs != gs) return false;
    rows += p->out;
  }
  std::vector<int8_t> q((size_t)rows * in);
  std::vector<float> s((size_t)rows * (in / gs));
  size_t oq = 0, os = 0;
  for (auto* p : parts) {
    memcpy(q.data() + oq, p->q.data(), p->q.size());
    memcpy(s.data() + os, p->s.data(), p->s.size() * 4);
    oq += p->q.size();
    os += p->s.size();
  }
  out->out = rows; out->in = in; out->gs = gs;
  out->q = dev_upload(m, q.data(), q.size());
  out->s = dev_upload(m, s.data(), s.size());
  return out->q && out->s;
}

bool up_one(LZModel* m, const HQ& h, QW* out) { return up_group(m, {&h}, out); }

}  // namespace

// ====================================================================== model

extern "C" int lz_open(LZModel** out, const char* dir, char* errbuf, int errlen) {
  if (!out || !dir) { set_err(errbuf, errlen, "null argument"); return LZ98_ERR_NULL_ARG; }
  *out = nullptr;
  std::string path = std::string(dir) + "/model.bin";
  Reader r;
  r.f = fopen(path.c_str(), "rb");
  if (!r.f) { set_err(errbuf, errlen, "cannot open %s", path.c_str()); return LZ98_ERR_MODEL; }
  LZModel* m = new LZModel();
  Cfg& c = m->c;
  cudaGetDevice(&m->dev);
  char magic[4];
  r.bytes(magic, 4);
  int ver = r.i32();
  if (memcmp(magic, "L98Z", 4) != 0 || ver < 5 || ver > 9) {
    set_err(errbuf, errlen, "not an L98Z v5-v9 model.bin");
    fclose(r.f); delete m; return LZ98_ERR_MODEL;
  }
  // Header words in the order of src/model.c:3993-4301.
  c.vocab = r.i32(); c.d = r.i32(); c.nl = r.i32(); c.seq_len = r.i32();
  c.nh = r.i32(); c.nkv = r.i32(); c.hd = r.i32(); c.inter = r.i32();
  c.nk = r.i32(); c.nv = r.i32(); c.kd = r.i32(); c.vd = r.i32();
  c.conv_k = r.i32(); r.i32(); r.i32(); r.i32(); r.i32(); r.i32();
  c.eps = r.f32(); c.theta = r.f32(); c.prf = r.f32();
  c.q_dim = r.i32(); c.qg_dim = r.i32(); c.kv_dim = r.i32();
  c.key_dim = r.i32(); c.val_dim = r.i32(); c.conv_dim = r.i32(); c.rot = r.i32();
  int lt[128];
  for (int i = 0; i < 128; i++) lt[i] = r.i32();
  c.rank = r.i32(); c.has_lb = r.i32(); c.lb = r.f32();
  c.ne = r.i32(); c.topk = r.i32(); c.n_shared = r.i32(); c.moe_ffn = r.i32();
  c.latent = r.i32(); c.fkdr = r.i32(); c.renorm = r.i32(); c.sigm = r.i32();
  c.lat_norm = r.i32(); c.shared_w = r.i32();
  c.mtp_layers = r.i32(); c.mtp_ffn = r.i32();
  for (int i = 0; i < 15; i++) r.i32();
  for (int i = 0; i < 3 * 128; i++) r.i32();
  for (int i = 0; i < 6; i++) r.i32();
  for (int i = 0; i < 128; i++) r.i32();
  // v6-v9 words (src/model.c:4352-4440): this path takes the identity
  // layer schedule, one MTP draft, no embedding rotation and no input
  // mixing or local attention window; any scale layout
  bool sched_ok = true;
  if (ver >= 6) {
    const int exec_len = r.i32();
    int app_layer[128], app_loop[128];
    for (int i = 0; i < 128; i++) app_layer[i] = r.i32();
    for (int i = 0; i < 128; i++) app_loop[i] = r.i32();
    const int n_draft = r.i32(), hadamard = r.i32();
    r.i32();   // embed_signs_seed
    r.layout = r.i32();
    sched_ok = exec_len == c.nl && n_draft <= 1 && hadamard == 0 && r.layout >= 0 && r.layout <= 2;
    for (int i = 0; i < 128 && sched_ok; i++)
      sched_ok = app_layer[i] == (i < c.nl ? i : 0) && app_loop[i] == 0;
  }
  if (ver >= 7 && r.i32() != 0) sched_ok = false;   // loop_input_mix
  if (ver >= 8 && r.i32() != 0) sched_ok = false;   // ced_local
  if (ver >= 9) r.i32();                            // loop_input_mix_from (unused without mixing)
  bool ok = !r.bad && sched_ok;
  for (int l = 0; l < c.nl && ok; l++) ok = lt[l] == 2;
  ok = ok && c.fkdr == 0 && c.ne > 0 && c.ne <= 256 && c.topk <= 16 && c.mtp_layers == 1 &&
       !c.lat_norm && c.has_lb && c.sigm && c.renorm && c.kd == 64 && c.vd == 64 &&
       c.nk == c.nv && c.hd == 64 && c.conv_k == 4 && c.d % 32 == 0 && c.rank % 32 == 0 &&
       c.rank <= 128 && c.latent <= 1024 && c.latent % 32 == 0 && c.moe_ffn % 32 == 0 &&
       c.shared_w % 32 == 0 && 2 * c.d <= 4096 && c.moe_ffn <= 2048 && c.val_dim <= 4096;
  if (!ok) {
    set_err(errbuf, errlen, "unsupported KunMoe configuration (needs all-KDA layers, latent MoE with "
                            "sigmoid router, one MTP layer, head dims 64)");
    fclose(r.f); delete m; return LZ98_ERR_MODEL;
  }
  HQ embed = r.qten(c.vocab, c.d);
  std::vector<float> fnorm = r.ften(c.d);
  if (!r.bad) {
    up_one(m, embed, &m->embed);
    m->final_norm = up_f(m, fnorm);
  }
  const int kdim = c.key_dim, vdim = c.val_dim, nvk = c.nv * c.kd;
  m->off_q = 0; m->off_k = kdim; m->off_v = 2 * kdim; m->off_g = 2 * kdim + vdim;
  m->off_fa = 2 * kdim + 2 * vdim; m->off_b = m->off_fa + c.rank; m->n_in = m->off_b + c.nv;
  m->off_router = 0; m->off_down = c.ne; m->off_shg = c.ne + c.latent;
  m->off_shu = m->off_shg + c.shared_w; m->n_moe = m->off_shu + c.shared_w;
  m->off_mq = 0; m->off_mk = c.qg_dim; m->off_mv = c.qg_dim + c.kv_dim;
  m->n_qkv = c.qg_dim + 2 * c.kv_dim;
  m->L.resize(c.nl);
  for (int l = 0; l < c.nl && !r.bad; l++) {
    DLayer& L = m->L[l];
    auto in_ln = r.ften(c.d), post_ln = r.ften(c.d);
    HQ q = r.qten(kdim, c.d), k = r.qten(kdim, c.d), v = r.qten(vdim, c.d);
    auto qc = r.ften((size_t)kdim * c.conv_k), kc = r.ften((size_t)kdim * c.conv_k),
         vc = r.ften((size_t)vdim * c.conv_k);
    auto a_log = r.ften(c.nv);
    HQ fa = r.qten(c.rank, c.d), fb = r.qten(nvk, c.rank);
    auto dt_bias = r.ften(nvk);
    HQ b = r.qten(c.nv, c.d), g = r.qten(vdim, c.d);
    auto o_norm = r.ften(c.vd);
    HQ o = r.qten(c.d, vdim);
    HQ router = r.qten(c.ne, c.d);
    auto rbias = r.ften(c.ne);
    HQ down = r.qten(c.latent, c.d), up = r.qten(c.d, c.latent);
    HQ shg, shu, shd;
    if (c.shared_w) {
      shg = r.qten(c.shared_w, c.d); shu = r.qten(c.shared_w, c.d); shd = r.qten(c.d, c.shared_w);
    }
    std::vector<int8_t> w13q, w2q;
    std::vector<float> w13s, w2s;
    int gs1 = 0, gs2 = 0;
    for (int e = 0; e < c.ne && !r.bad; e++) {
      HQ w1 = r.qten(c.moe_ffn, c.latent), w2 = r.qten(c.latent, c.moe_ffn), w3 = r.qten(c.moe_ffn, c.latent);
      if (r.bad) break;
      if (e == 0) { gs1 = w1.gs; gs2 = w2.gs; }
      if (w1.gs != gs1 || w3.gs != gs1 || w2.gs != gs2) { r.bad = true; break; }
      w13q.insert(w13q.end(), w1.q.begin(), w1.q.end());
      w13q.insert(w13q.end(), w3.q.begin(), w3.q.end());
      w13s.insert(w13s.end(), w1.s.begin(), w1.s.end());
      w13s.insert(w13s.end(), w3.s.begin(), w3.s.end());
      w2q.insert(w2q.end(), w2.q.begin(), w2.q.end());
      w2s.insert(w2s.end(), w2.s.begin(), w2.s.end());
    }
    if (r.bad) break;
    std::vector<float> conv_w;
    conv_w.insert(conv_w.end(), qc.begin(), qc.end());
    conv_w.insert(conv_w.end(), kc.begin(), kc.end());
    conv_w.insert(conv_w.end(), vc.begin(), vc.end());
    L.in_ln = up_f(m, in_ln); L.post_ln = up_f(m, post_ln); L.conv_w = up_f(m, conv_w);
    L.a_log = up_f(m, a_log); L.dt_bias = up_f(m, dt_bias); L.o_norm = up_f(m, o_norm);
    L.router_bias = up_f(m, rbias);
    bool g_ok = up_group(m, {&q, &k, &v, &g, &fa, &b}, &L.inproj) && up_one(m, fb, &L.fb) &&
                up_one(m, o, &L.o) && up_one(m, up, &L.up);
    if (c.shared_w) {
      g_ok = g_ok && up_group(m, {&router, &down, &shg, &shu}, &L.moein) && up_one(m, shd, &L.sh_down);
    } else {
      g_ok = g_ok && up_group(m, {&router, &down}, &L.moein);
    }
    L.w13q = dev_upload(m, w13q.data(), w13q.size());
    L.w13s = dev_upload(m, w13s.data(), w13s.size());
    L.w2q = dev_upload(m, w2q.data(), w2q.size());
    L.w2s = dev_upload(m, w2s.data(), w2s.size());
    L.w13_gs = gs1; L.w2_gs = gs2;
    if (!g_ok) { r.bad = true; break; }
  }
  if (!r.bad) {
    DMtp& M = m->mtp;
    auto in_ln = r.ften(c.d), post_ln = r.ften(c.d);
    HQ qp = r.qten(c.qg_dim, c.d), kp = r.qten(c.kv_dim, c.d), vp = r.qten(c.kv_dim, c.d);
    HQ op = r.qten(c.d, c.q_dim);
    auto qn = r.ften(c.hd), kn = r.ften(c.hd);
    HQ gate = r.qten(c.mtp_ffn, c.d), up = r.qten(c.mtp_ffn, c.d), down = r.qten(c.d, c.mtp_ffn);
    HQ fc = r.qten(c.d, 2 * c.d);
    auto norm = r.ften(c.d), pre_h = r.ften(c.d), pre_e = r.ften(c.d);
    if (!r.bad) {
      M.in_ln = up_f(m, in_ln); M.post_ln = up_f(m, post_ln); M.q_norm = up_f(m, qn);
      M.k_norm = up_f(m, kn); M.norm = up_f(m, norm); M.pre_h = up_f(m, pre_h); M.pre_e = up_f(m, pre_e);
      bool g_ok = up_group(m, {&qp, &kp, &vp}, &M.qkv) && up_one(m, op, &M.o) &&
                  up_group(m, {&gate, &up}, &M.gu) && up_one(m, down, &M.down) && up_one(m, fc, &M.fc);
      if (!g_ok) r.bad = true;
    }
  }
  fclose(r.f);
  if (r.bad) {
    set_err(errbuf, errlen, "truncated or malformed model.bin (or mixed group sizes in a fused group)");
    lz_free(m);
    return LZ98_ERR_MODEL;
  }
  if (cudaDeviceSynchronize() != cudaSuccess) {
    set_err(errbuf, errlen, "CUDA failure while uploading weights");
    lz_free(m);
    return LZ98_ERR_CUDA;
  }
  *out = m;
  return 0;
}

// The reference reads the tensors in a second call after lz_open
// (src/model.h:1333-1339); here lz_open already uploaded them to HBM, so
// this only checks the handle.
extern "C" int lz_read_weights(LZModel* m, char* errbuf, int errlen) {
  if (!m) {
    set_err(errbuf, errlen, "null argument");
    return LZ98_ERR_NULL_ARG;
  }
  return 0;
}

extern "C" void lz_free(LZModel* m) {
  if (!m) return;
  for (void* p : m->allocs) cudaFree(p);
  delete m;
}

extern "C" void lz_model_info(const LZModel* m, int* o) {
  const Cfg& c = m->c;
  int v[16] = {c.vocab, c.d, c.nl, c.nv, c.key_dim, c.latent, c.ne, c.topk, c.shared_w,
               c.hd, c.nh, c.nkv, c.rot, c.seq_len, c.mtp_ffn, c.moe_ffn};
  memcpy(o, v, sizeof v);
}

extern "C" size_t lz_model_weight_bytes(const LZModel* m) { return m ? m->wbytes : 0; }

// ======================================================================= NCCL
//
// Expert parallelism exchanges pairs with NCCL send/recv.  The library is
// bound at run time: the NCCL a host process already loaded (a PyTorch
// process has one) is reused, else libnccl.so.2 is opened; nothing links
// against it, so one-GPU use needs no NCCL at all.
namespace {
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*comm_abort)(ncclComm_t);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  const char* (*error_string)(ncclResult_t);
};

const NcclApi* nccl_api() {
  static std::once_flag once;
  static NcclApi api;
  static bool ok = false;
  std::call_once(once, [] {
    // the NCCL already in the process (a framework's), else LZ98_NCCL (a
    // path), else the system's.  A process that loads another NCCL later
    // must load it first: a second library of the same soname is not
    // loaded beside this one.
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) {
      const char* path = getenv("LZ98_NCCL");
      if (path && *path) h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    }
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    auto take = [h](auto& fn, const char* name) {
      void* p = dlsym(h, name);
      memcpy(&fn, &p, sizeof p);
      return p != nullptr;
    };
    ok = take(api.get_unique_id, "ncclGetUniqueId") && take(api.comm_init_rank, "ncclCommInitRank") &&
         take(api.comm_destroy, "ncclCommDestroy") && take(api.comm_abort, "ncclCommAbort") &&
         take(api.group_start, "ncclGroupStart") && take(api.group_end, "ncclGroupEnd") &&
         take(api.send, "ncclSend") && take(api.recv, "ncclRecv") && take(api.error_string, "ncclGetErrorString");
  });
  return ok ? &api : nullptr;
}

// Expert-parallel context of a run state (lz_ep_init): communicator, the
// owned expert range, the slot buffers and the per-layer scratch.
struct EpCtx {
  int world = 1, rank = 0, epr = 0, e0 = 0;
  ncclComm_t comm = nullptr;
  EpBuf buf{};
  int *pair_dest = nullptr, *pair_slot = nullptr;       // per local pair: owner, slot
  int *expert = nullptr, *src = nullptr, *slot = nullptr, *total = nullptr;   // per received pair
  int *list = nullptr, *ntiles = nullptr;
  MoeTile* tiles = nullptr;
  int8_t *latq = nullptr, *hq = nullptr;
  float *lats = nullptr, *hs = nullptr, *h2 = nullptr, *sendback = nullptr, *recvback = nullptr;
  bool failed = false;                                   // an exchange failed or timed out
};
constexpr double kEpTimeoutS = 60.0;   // a stream of an expert-parallel state that has not drained by then is aborted
}  // namespace

// ====================================================================== state

struct LZRunState {
  const LZModel* m = nullptr;
  int B = 1, seq_len = 0, depth = 1, kmax = 1, Rmax = 64;
  cudaStream_t st = nullptr;
  // recurrent state and caches
  int8_t *hi = nullptr, *lo = nullptr;
  float *sc = nullptr, *conv = nullptr;
  int8_t *kq = nullptr, *vq = nullptr;
  float *ks = nullptr, *vs = nullptr, *chain = nullptr, *rope = nullptr;
  size_t q_slot = 0, q_seq = 0, conv_slot = 0, conv_seq = 0, cache_seq = 0;
  float attn_scale = 0, ssm_scale = 0;
  // scratch
  float *x, *inproj, *moein, *h2, *shout, *hidden, *logits, *qkv, *mtpx, *hb;
  int8_t *xq, *oq, *latq, *hq, *yq, *shq, *aq;
  float *xs, *os, *lats, *hs, *ys, *shs, *as;
  int *pair_e, *tok, *catch_tok, *catch_hidx;
  unsigned long long* vmax;
  int* row_counter;                  // last-block tails per (row, 32-group) (reset by the last block)
  int* accept_counter;               // the fused greedy tail's block count (reset by its last block)
  // temperature rounds: draft distributions [B][kmax][V], target
  // distributions [Rmax][V], sort scratch [Rmax][npow2], sampled token
  float *qbuf = nullptr, *pbuf = nullptr, *sortbuf = nullptr;
  int npow2 = 2;
  int* tok_out = nullptr;
  // grouped experts: pair indices by expert, tiles, tile count
  int* glist = nullptr;
  MoeTile* gtiles = nullptr;
  int* gntiles = nullptr;
  std::vector<char> seq_temp;        // per sequence: temperature mode
  int n_sm = 148;
  std::map<long, int> gemv_occ;      // resident GEMV blocks per SM by (JM, shared bytes)
  float* pair_w;
  KdaSeq* seqs;
  MtpRow *mrows, *crows;
  SeqRound* sr;
  size_t hb_rows = 0;
  // host mirrors
  std::vector<SeqRound> h_sr;
  std::vector<float> h_logits, h_hidden, h_draft;
  long long launches = 0;
  bool graphs = true;
  bool pdl = true;                   // programmatic dependent launch
  bool umma = false;                 // R > 8 dense GEMMs on tcgen05 (else the mma.sync TMA kernel)
  // optional per-GEMV timing (lz_profile_round): event pairs and bytes
  bool prof = false;
  std::vector<cudaEvent_t> prof_ev;
  std::vector<double> prof_bytes;
  // and per grouped-expert launch (lz_profile_experts): event pairs, bytes
  std::vector<cudaEvent_t> prof_moe_ev;
  std::vector<double> prof_moe_bytes;
  double prof_moe_ms = 0.0, prof_moe_b = 0.0;
  int prof_moe_n = 0;
  // optional per-launch timing (lz_profile_launches): kernel and event pair
  bool prof_all = false;
  std::vector<std::tuple<const void*, cudaEvent_t, cudaEvent_t>> prof_launch;
  std::map<int, cudaGraphExec_t> graph;
  std::vector<void*> allocs;
  // 1 at allocation, +1 per reset (src/forward_state.c:1412,
  // src/forward.c:782); a checkpoint records it and restore refuses a change
  unsigned epoch = 1;
  // TMA descriptors of the staged GEMM by (base, inner extent, rows, box
  // inner, box rows); built on first use, baked into captured graphs
  std::map<std::tuple<const void*, int, int, int, int>, CUtensorMap> tmaps;
  // device-side error word in mapped pinned memory: set by a kernel whose
  // bounded wait gave up; read after every synchronisation
  int* h_err = nullptr;
  int* d_err = nullptr;
  float* pconf = nullptr;            // confidence of a p_min draft step
  EpCtx ep;                          // expert parallelism (lz_ep_init)
  bool dbg_timing = false;           // events around the parts of a round
  cudaEvent_t dbg_ev[4] = {nullptr, nullptr, nullptr, nullptr};
};

// Wait for the state's stream; false on a CUDA error or when a kernel
// reported a wait that gave up (the error word stays set until the state
// is freed: the run state is then not trustworthy).
static bool sync_ok(const LZRunState* cs) {
  LZRunState* s = const_cast<LZRunState*>(cs);
  if (s->ep.comm) {
    // an expert-parallel stream waits on its peers: poll it with a deadline
    // and abort the communicator (its kernels then return) if it passes
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      const cudaError_t q = cudaStreamQuery(s->st);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) return false;
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > kEpTimeoutS) {
        if (const NcclApi* n = nccl_api()) n->comm_abort(s->ep.comm);
        s->ep.comm = nullptr;
        s->ep.failed = true;
        return false;
      }
      usleep(20);
    }
    if (s->ep.failed) return false;
  } else if (cudaStreamSynchronize(s->st) != cudaSuccess) {
    return false;
  }
  return !(s->h_err && *(volatile int*)s->h_err);
}

namespace {

// Every kernel of the forward and the round is launched through here: with
// programmatic stream serialisation when enabled, so the next kernel's
// prologue (weight prefetch) overlaps this one's tail.
template <typename... KArgs, typename... Args>
void launch(LZRunState* s, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s->st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // debug timing puts event records between kernels: plain launches then
  cfg.numAttrs = s->pdl && !s->dbg_timing && !s->prof_all ? 1 : 0;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (s->prof_all && cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess)
    cudaEventRecord(e0, s->st);
  cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e1) {
    cudaEventRecord(e1, s->st);
    s->prof_launch.emplace_back((const void*)kern, e0, e1);
  }
  s->launches++;
}

// Every TMA GEMM variant the launcher uses, with its dynamic shared memory
// (the limit is raised for each at state allocation).
template <typename F>
void tma_variants(F f) {
  f(gemm_q8_tma_kernel<1, 1, true, 0>, TmaTile<1, 1, true>::smem());
  f(gemm_q8_tma_kernel<1, 2, true, 0>, TmaTile<1, 2, true>::smem());
  f(gemm_q8_tma_kernel<2, 1, true, 0>, TmaTile<2, 1, true>::smem());
  f(gemm_q8_tma_kernel<1, 1, false, 1>, TmaTile<1, 1, false>::smem());
  f(gemm_q8_tma_kernel<1, 2, false, 1>, TmaTile<1, 2, false>::smem());
  f(gemm_q8_tma_kernel<2, 1, false, 1>, TmaTile<2, 1, false>::smem());
  f(gemm_q8_tma_kernel<1, 1, false, 2>, TmaTile<1, 1, false>::smem());
  f(gemm_q8_tma_kernel<1, 2, false, 2>, TmaTile<1, 2, false>::smem());
  f(gemm_q8_tma_kernel<2, 1, false, 2>, TmaTile<2, 1, false>::smem());
  f(gemm_q8_umma_kernel<16, 0>, UmmaTile<16, true>::smem());
  f(gemm_q8_umma_kernel<16, 1>, UmmaTile<16, false>::smem());
  f(gemm_q8_umma_kernel<16, 2>, UmmaTile<16, false>::smem());
  f(moe_tma_kernel<true, true, 0>, MoeTma<true, true>::smem(MoeTma<true, true>::KMAX));
  f(moe_tma_kernel<true, false, 1>, MoeTma<true, false>::smem(MoeTma<true, false>::KMAX));
  f(moe_tma_kernel<true, false, 2>, MoeTma<true, false>::smem(MoeTma<true, false>::KMAX));
  f(moe_tma_kernel<false, true, 0>, MoeTma<false, true>::smem(MoeTma<false, true>::KMAX));
  f(moe_tma_kernel<false, false, 1>, MoeTma<false, false>::smem(MoeTma<false, false>::KMAX));
  f(moe_tma_kernel<false, false, 2>, MoeTma<false, false>::smem(MoeTma<false, false>::KMAX));
}

template <typename T>
bool dmalloc(LZRunState* s, T** p, size_t n) {
  if (cudaMalloc((void**)p, n * sizeof(T) + 64) != cudaSuccess) return false;
  cudaMemset(*p, 0, n * sizeof(T) + 64);
  s->allocs.push_back(*p);
  return true;
}

// RoPE table (src/forward_rope.c:178-187, no scaling), with the
// reference's own float pow / cos / sin restated in lz98_rope_table.h.
void build_rope(const Cfg& c, int seq_len, std::vector<float>& t) {
  t.assign((size_t)seq_len * c.rot, 0.0f);
  lz98_rope_table(c.theta, c.rot, seq_len, t.data());
}

float host_rsqrt_body(float x) {         // src/ops_quant.c:126-135
  union { float f; uint32_t u; } t;
  volatile float h = 0.5f * x;
  float y;
  t.f = x;
  t.u = 0x5f375a86u - (t.u >> 1);
  y = t.f;
  volatile float a = h * y;
  volatile float b = a * y;
  volatile float cc = 1.5f - b;
  y = y * cc;
  a = h * y; b = a * y; cc = 1.5f - b;
  y = y * cc;
  return y;
}

}  // namespace

static int state_alloc(LZRunState** out, const LZModel* m, int n_seq, int seq_len, int spec_k_max,
                       char* errbuf, int errlen) {
  if (!out || !m || n_seq < 1 || seq_len < 2 || spec_k_max < 1 || spec_k_max > 6) {
    set_err(errbuf, errlen, "bad state arguments");
    return LZ98_ERR_NULL_ARG;
  }
  const Cfg& c = m->c;
  LZRunState* s = new LZRunState();
  s->m = m;
  s->B = n_seq;
  s->seq_len = seq_len;
  s->depth = spec_k_max + 1;              // src/forward_state.c:738-744
  s->kmax = spec_k_max;
  s->Rmax = std::max(64, n_seq * (spec_k_max + 1));
  if ((long)s->Rmax * m->c.topk > 1024L * kMoeGroupPer) {
    set_err(errbuf, errlen, "too many sequences for one forward (rows x top-k above the expert grouping's limit)");
    delete s;
    return LZ98_ERR_SIZE;
  }
  if (cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking) != cudaSuccess) {
    delete s;
    set_err(errbuf, errlen, "cudaStreamCreate failed");
    return LZ98_ERR_CUDA;
  }
  if (cudaHostAlloc((void**)&s->h_err, sizeof(int), cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer((void**)&s->d_err, s->h_err, 0) != cudaSuccess) {
    set_err(errbuf, errlen, "cannot map the device error word");
    lz_state_free(s);
    return LZ98_ERR_ALLOC;
  }
  *s->h_err = 0;
  s->q_slot = (size_t)c.nl * c.nv * c.kd * c.vd;
  s->q_seq = s->q_slot * s->depth;
  s->conv_slot = (size_t)c.nl * c.conv_dim * 3;
  s->conv_seq = s->conv_slot * s->depth;
  s->cache_seq = (size_t)seq_len * c.kv_dim;
  const size_t B = n_seq, R = s->Rmax, P = R * c.topk;
  const int kmaxw = std::max({2 * c.d, c.key_dim, c.val_dim, c.moe_ffn, c.shared_w, c.latent, c.q_dim,
                              c.mtp_ffn, c.rank});
  const int nwide = std::max({m->n_in, m->n_moe, m->n_qkv, 2 * c.mtp_ffn});
  bool ok = dmalloc(s, &s->hi, s->q_seq * B) && dmalloc(s, &s->lo, s->q_seq * B) &&
            dmalloc(s, &s->sc, s->q_seq * B / 32) && dmalloc(s, &s->conv, s->conv_seq * B) &&
            dmalloc(s, &s->kq, s->cache_seq * B) && dmalloc(s, &s->vq, s->cache_seq * B) &&
            dmalloc(s, &s->ks, s->cache_seq * B / 32) && dmalloc(s, &s->vs, s->cache_seq * B / 32) &&
            dmalloc(s, &s->chain, B * c.d) && dmalloc(s, &s->rope, (size_t)seq_len * c.rot) &&
            dmalloc(s, &s->x, R * c.d) && dmalloc(s, &s->inproj, R * nwide) &&
            dmalloc(s, &s->moein, R * m->n_moe) && dmalloc(s, &s->h2, P * c.latent) &&
            dmalloc(s, &s->shout, R * c.d) && dmalloc(s, &s->hidden, R * c.d) &&
            dmalloc(s, &s->logits, R * (size_t)c.vocab) && dmalloc(s, &s->qkv, R * m->n_qkv) &&
            dmalloc(s, &s->mtpx, R * c.d) && dmalloc(s, &s->xq, R * kmaxw) &&
            dmalloc(s, &s->xs, R * kmaxw / 32) && dmalloc(s, &s->oq, R * c.val_dim) &&
            dmalloc(s, &s->os, R * c.val_dim / 32) && dmalloc(s, &s->latq, R * c.latent) &&
            dmalloc(s, &s->lats, R * c.latent / 32) && dmalloc(s, &s->hq, P * c.moe_ffn) &&
            dmalloc(s, &s->hs, P * c.moe_ffn / 32) && dmalloc(s, &s->yq, R * c.latent) &&
            dmalloc(s, &s->ys, R * c.latent / 32) &&
            dmalloc(s, &s->shq, R * std::max(c.shared_w, c.mtp_ffn)) &&
            dmalloc(s, &s->shs, R * std::max(c.shared_w, c.mtp_ffn) / 32) &&
            dmalloc(s, &s->aq, R * c.q_dim) && dmalloc(s, &s->as, R * c.q_dim / 32) &&
            dmalloc(s, &s->pair_e, P) && dmalloc(s, &s->pair_w, P) && dmalloc(s, &s->tok, R) &&
            dmalloc(s, &s->vmax, R) && dmalloc(s, &s->catch_tok, R) && dmalloc(s, &s->catch_hidx, R) &&
            dmalloc(s, &s->seqs, R) && dmalloc(s, &s->mrows, R) && dmalloc(s, &s->crows, R) &&
            dmalloc(s, &s->sr, B) && dmalloc(s, &s->row_counter, R * (c.latent / 32 + 1)) && dmalloc(s, &s->accept_counter, 1) && dmalloc(s, &s->tok_out, 4) &&
            dmalloc(s, &s->pconf, 4);
  s->npow2 = 2;
  while (s->npow2 < c.vocab) s->npow2 <<= 1;
  ok = ok && dmalloc(s, &s->glist, P) && dmalloc(s, &s->gtiles, P / kMoeTileRows + std::min((size_t)c.ne, P) + 1) &&
       dmalloc(s, &s->gntiles, 1);
  ok = ok && dmalloc(s, &s->qbuf, B * s->kmax * (size_t)c.vocab) && dmalloc(s, &s->pbuf, R * (size_t)c.vocab) &&
       dmalloc(s, &s->sortbuf, R * 2 * (size_t)s->npow2);
  s->seq_temp.assign(B, 0);
  if (!ok) {
    set_err(errbuf, errlen, "device allocation failed");
    lz_state_free(s);
    return LZ98_ERR_ALLOC;
  }
  {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&s->n_sm, cudaDevAttrMultiProcessorCount, dev);
    // the GEMV input-norm prologue stages its rows in dynamic shared memory
    const int gdyn = 160 * 1024;
    auto attr = [gdyn](auto kern) {
      return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gdyn) == cudaSuccess;
    };
    bool tma_ok = true;
    tma_variants([&](auto kern, size_t bytes) {
      tma_ok = tma_ok && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess;
    });
    if (!tma_ok) {
      set_err(errbuf, errlen, "cannot raise the TMA GEMM shared-memory limit");
      lz_state_free(s);
      return LZ98_ERR_CUDA;
    }
    if (!attr(gemv_q8_kernel<1, kGemvProWarps, 1, true, false>) || !attr(gemv_q8_kernel<1, kGemvProWarps, 4, true, false>) ||
        !attr(gemv_q8_kernel<1, kGemvProWarps, 8, true, false>) || !attr(gemv_q8_kernel<2, kGemvProWarps, 1, true, false>) ||
        !attr(gemv_q8_kernel<2, kGemvProWarps, 4, true, false>) || !attr(gemv_q8_kernel<2, kGemvProWarps, 8, true, false>)) {
      set_err(errbuf, errlen, "cannot raise the GEMV shared-memory limit");
      lz_state_free(s);
      return LZ98_ERR_CUDA;
    }
  }
  {
    // the attention kernel keeps one score per cached position in dynamic
    // shared memory; lift the default 48 KiB cap when the cache is long
    const int dyn = seq_len * (int)sizeof(float);
    if (dyn > 24 * 1024 &&
        cudaFuncSetAttribute(mtp_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) != cudaSuccess) {
      set_err(errbuf, errlen, "sequence too long for the attention kernel's shared memory");
      lz_state_free(s);
      return LZ98_ERR_ALLOC;
    }
    // the MTP front keeps its two rows and their squares: 4 d + 32 floats
    const int front = (4 * m->c.d + 32) * (int)sizeof(float);
    if (front > 48 * 1024 &&
        cudaFuncSetAttribute(mtp_front_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, front) != cudaSuccess) {
      set_err(errbuf, errlen, "hidden size too large for the MTP front kernel's shared memory");
      lz_state_free(s);
      return LZ98_ERR_ALLOC;
    }
  }
  std::vector<float> rope;
  build_rope(c, seq_len, rope);
  cudaMemcpy(s->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice);
  s->attn_scale = host_rsqrt_body((float)c.hd);     // src/forward_state.c:1408-1409
  s->ssm_scale = host_rsqrt_body((float)c.kd);
  s->h_sr.assign(B, SeqRound{});
  s->h_logits.resize((size_t)R * c.vocab);
  s->h_hidden.resize((size_t)R * c.d);
  s->h_draft.resize(c.vocab);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    set_err(errbuf, errlen, "CUDA failure in state allocation");
    lz_state_free(s);
    return LZ98_ERR_CUDA;
  }
  *out = s;
  return 0;
}

extern "C" int lz_state_alloc(LZRunState** out, const LZModel* m, int seq_len, int spec_k_max,
                              char* errbuf, int errlen) {
  return state_alloc(out, m, 1, seq_len, spec_k_max, errbuf, errlen);
}

extern "C" int lz_state_alloc_batch(LZRunState** out, const LZModel* m, int n_seq, int seq_len,
                                    int spec_k_max, char* errbuf, int errlen) {
  return state_alloc(out, m, n_seq, seq_len, spec_k_max, errbuf, errlen);
}

extern "C" void lz_state_free(LZRunState* s) {
  if (!s) return;
  if (s->ep.comm) {
    const bool drained = sync_ok(s);    // aborts the communicator itself when the stream does not drain
    if (const NcclApi* n = nccl_api()) {
      if (drained && s->ep.comm) n->comm_destroy(s->ep.comm);
      else if (s->ep.comm) n->comm_abort(s->ep.comm);
    }
    s->ep.comm = nullptr;
  }
  for (auto& kv : s->graph) cudaGraphExecDestroy(kv.second);
  for (void* p : s->allocs) cudaFree(p);
  if (s->h_err) cudaFreeHost(s->h_err);
  for (auto e : s->dbg_ev)
    if (e) cudaEventDestroy(e);
  if (s->st) cudaStreamDestroy(s->st);
  delete s;
}

static void clear_state(LZRunState* s) {
  const Cfg& c = s->m->c;
  const size_t B = s->B;
  cudaMemsetAsync(s->hi, 0, s->q_seq * B, s->st);
  cudaMemsetAsync(s->lo, 0, s->q_seq * B, s->st);
  cudaMemsetAsync(s->sc, 0, s->q_seq * B / 32 * 4, s->st);
  cudaMemsetAsync(s->conv, 0, s->conv_seq * B * 4, s->st);
  cudaMemsetAsync(s->kq, 0, s->cache_seq * B, s->st);
  cudaMemsetAsync(s->vq, 0, s->cache_seq * B, s->st);
  cudaMemsetAsync(s->ks, 0, s->cache_seq * B / 32 * 4, s->st);
  cudaMemsetAsync(s->vs, 0, s->cache_seq * B / 32 * 4, s->st);
  cudaMemsetAsync(s->chain, 0, B * c.d * 4, s->st);
  // the sampler (temperature, top-p, generator) is not part of the run
  // state in the reference (LZSampler, src/sampler.h:145-187): kept
  cudaMemcpyAsync(s->h_sr.data(), s->sr, B * sizeof(SeqRound), cudaMemcpyDeviceToHost, s->st);
  cudaStreamSynchronize(s->st);
  for (auto& r : s->h_sr) {
    SeqRound z{};
    z.rng = r.rng;
    z.temp = r.temp;
    z.topp = r.topp;
    r = z;
  }
  cudaMemcpyAsync(s->sr, s->h_sr.data(), B * sizeof(SeqRound), cudaMemcpyHostToDevice, s->st);
  cudaStreamSynchronize(s->st);
}

extern "C" void lz_state_reset(LZRunState* s, const LZModel*) {
  if (!s) return;
  clear_state(s);
  s->epoch++;
}

// Round records device -> host (waits for the stream) and host -> device
// (queued); false on a CUDA failure or, for sr_down, a device wait that
// gave up (sync_ok).
static bool sr_down(LZRunState* s) {
  return cudaMemcpyAsync(s->h_sr.data(), s->sr, s->B * sizeof(SeqRound), cudaMemcpyDeviceToHost, s->st) ==
             cudaSuccess &&
         sync_ok(s);
}
static bool sr_up(LZRunState* s) {
  return cudaMemcpyAsync(s->sr, s->h_sr.data(), s->B * sizeof(SeqRound), cudaMemcpyHostToDevice, s->st) ==
         cudaSuccess;
}

// errbuf text of a failed device round: a bounded device wait that gave up
// (the state's error word) or the CUDA error.
static void round_fail(const LZRunState* s, char* errbuf, int errlen, const char* what) {
  const cudaError_t e = cudaGetLastError();
  char msg[200];
  if (s->h_err && *(volatile int*)s->h_err)
    snprintf(msg, sizeof msg, "%s: a device wait gave up (the state is not usable)", what);
  else
    snprintf(msg, sizeof msg, "%s: %s", what, cudaGetErrorString(e));
  set_err(errbuf, errlen, "%s", msg);
}

extern "C" int lz_state_get(const LZRunState* cs, int seq, int* mtp_pos, int* ssm_slot, int* depth) {
  LZRunState* s = const_cast<LZRunState*>(cs);
  if (!s || seq < 0 || seq >= s->B) return LZ98_ERR_NULL_ARG;
  if (!sr_down(s)) return LZ98_ERR_CUDA;
  if (mtp_pos) *mtp_pos = s->h_sr[seq].mtp_pos;
  if (ssm_slot) *ssm_slot = s->h_sr[seq].ssm_slot;
  if (depth) *depth = s->depth;
  return 0;
}

extern "C" int lz_state_set(LZRunState* s, int seq, int mtp_pos, int ssm_slot) {
  if (!s || seq < 0 || seq >= s->B) return LZ98_ERR_NULL_ARG;
  if (!sr_down(s)) return LZ98_ERR_CUDA;
  if (mtp_pos >= 0) s->h_sr[seq].mtp_pos = mtp_pos;
  if (ssm_slot >= 0) s->h_sr[seq].ssm_slot = ssm_slot % s->depth;
  return sr_up(s) && sync_ok(s) ? 0 : LZ98_ERR_CUDA;
}

extern "C" int lz_state_get_chain(const LZRunState* s, int seq, float* chain) {
  if (!s || !chain || seq < 0 || seq >= s->B) return LZ98_ERR_NULL_ARG;
  const int d = s->m->c.d;
  cudaMemcpyAsync(chain, s->chain + (size_t)seq * d, d * 4, cudaMemcpyDeviceToHost, s->st);
  return sync_ok(s) ? 0 : LZ98_ERR_CUDA;
}

extern "C" int lz_state_set_chain(LZRunState* s, int seq, const float* chain) {
  if (!s || !chain || seq < 0 || seq >= s->B) return LZ98_ERR_NULL_ARG;
  const int d = s->m->c.d;
  cudaMemcpyAsync(s->chain + (size_t)seq * d, chain, d * 4, cudaMemcpyHostToDevice, s->st);
  return sync_ok(s) ? 0 : LZ98_ERR_CUDA;
}

extern "C" void* lz_state_stream(LZRunState* s) { return s ? (void*)s->st : nullptr; }
extern "C" long long lz_state_launches(const LZRunState* s) { return s ? s->launches : 0; }
extern "C" int lz_set_graphs(LZRunState* s, int enable) {
  if (!s) return LZ98_ERR_NULL_ARG;
  s->graphs = enable != 0 && !s->ep.comm;   // expert-parallel rounds run eagerly
  return 0;
}

extern "C" int lz_set_umma(LZRunState* s, int enable) {
  if (!s) return LZ98_ERR_NULL_ARG;
  if (s->umma != (enable != 0)) {
    for (auto& kv : s->graph) cudaGraphExecDestroy(kv.second);
    s->graph.clear();
  }
  s->umma = enable != 0;
  return 0;
}

extern "C" int lz_set_pdl(LZRunState* s, int enable) {
  if (!s) return LZ98_ERR_NULL_ARG;
  if (s->pdl != (enable != 0)) {
    for (auto& kv : s->graph) cudaGraphExecDestroy(kv.second);
    s->graph.clear();
  }
  s->pdl = enable != 0;
  return 0;
}

// ================================================================== launches

namespace {

// RMSNorm of a GEMV's input rows: the float rows (ld = the GEMV's K), the
// norm weights, an optional float copy of the normalised rows and optional
// arg-max slots to clear.
struct InNorm {
  const float* x;
  const float* w;
  float* out;
  unsigned long long* amax;
};

constexpr int kPrologueRows = 8;    // above this the norm runs as its own grid
constexpr int kGemvMaxBlocksPerSM = 16;

void rmsnorm_quant(LZRunState* s, const float* x, int ldx, const float* w, int n, int R, float* out,
                   int ldo, int8_t* xq, float* xs, unsigned long long* amax_clear = nullptr);

template <int JM, int WARPS, int RB, bool PRO, bool SINGLE>
void gemv_launch(LZRunState* s, const GemvArgs& a) {
  const size_t dyn = gemv_smem_bytes(JM, WARPS, RB, SINGLE, PRO, a.R, a.K);
  const long key = (long)JM << 56 | (long)WARPS << 48 | (long)RB << 44 | (long)PRO << 43 | (long)SINGLE << 42 |
                   (long)dyn;
  auto it = s->gemv_occ.find(key);
  int per_sm;
  if (it == s->gemv_occ.end()) {
    per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_q8_kernel<JM, WARPS, RB, PRO, SINGLE>, WARPS * 32,
                                                  dyn);
    per_sm = std::max(1, std::min(per_sm, kGemvMaxBlocksPerSM));
    s->gemv_occ[key] = per_sm;
  } else {
    per_sm = it->second;
  }
  const int want = (a.N + WARPS - 1) / WARPS;
  // a prologue is paid once per block: one block per SM
  const int cap = s->n_sm * (PRO ? 1 : per_sm);
  launch(s, gemv_q8_kernel<JM, WARPS, RB, PRO, SINGLE>, dim3(std::min(want, cap)), dim3(WARPS * 32), dyn, a);
}

template <int JM, int WARPS, bool PRO>
void gemv_launch_rb(LZRunState* s, const GemvArgs& a) {
  if (a.R <= 1) gemv_launch<JM, WARPS, 1, PRO, false>(s, a);
  else if (a.R <= 4) gemv_launch<JM, WARPS, 4, PRO, false>(s, a);
  else gemv_launch<JM, WARPS, 8, PRO, false>(s, a);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
PFN_cuTensorMapEncodeTiled_v12000 tma_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// The 2-D TMA map of a row-major operand, cached per state: int8 rows of
// `inner` bytes in 128-byte boxes with the 128-byte swizzle (box_inner
// 128), or f32 rows of `inner` floats in 16-byte boxes (box_inner 4).
// Rows past `rows` read as zeros.
const CUtensorMap* tmap(LZRunState* s, const void* base, int inner, int rows, int box_inner, int box_rows) {
  const auto key = std::make_tuple(base, inner, rows, box_inner, box_rows);
  auto it = s->tmaps.find(key);
  if (it != s->tmaps.end()) return &it->second;
  auto enc = tma_encoder();
  if (!enc) return nullptr;
  const bool f32 = box_inner == 4;
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t stride[1] = {(cuuint64_t)inner * (f32 ? 4 : 1)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows}, es[2] = {1, 1};
  if (enc(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
          stride, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, f32 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return nullptr;
  return &(s->tmaps[key] = m);
}

template <int MT, int NT, bool RB1, int GM>
void tma_launch(LZRunState* s, const GemmTmaArgs& a) {
  using T = TmaTile<MT, NT, RB1>;
  launch(s, gemm_q8_tma_kernel<MT, NT, RB1, GM>, dim3((a.N + T::BN - 1) / T::BN, (a.R + T::BM - 1) / T::BM), dim3(288),
         T::smem(), a);
}

// Grouped w1/w3 (w13) or w2 of one layer on the TMA-staged expert kernel;
// false when the shapes do not fit it (K % 128, K > 1024, output chunks).
// The expert shapes the TMA-staged kernels take (K % 128, K <= 1024,
// output chunks of 128 for both products).
bool moe_tma_fits(const Cfg& c) {
  return c.latent % 128 == 0 && c.moe_ffn % 128 == 0 && c.latent <= MoeTma<true, true>::KMAX &&
         c.moe_ffn <= MoeTma<true, true>::KMAX;
}

// Operands of the grouped expert kernels: the pairs (expert per pair,
// relative to the first expert e0 of ne), the grouping scratch, the
// activation rows (pair p reads latent row p / topk) and the outputs.
struct MoeIO {
  const int* pair_e; int P, topk, ne, e0;
  int* list; MoeTile* tiles; int* ntiles;
  const int8_t* latq; const float* lats;
  int8_t* hq; float* hs; float* h2;
};

bool moe_tma(LZRunState* s, bool w13, const int8_t* wq0, const float* wsc0, int gs, int tmax, const MoeIO& io) {
  const Cfg& c = s->m->c;
  const int K = w13 ? c.latent : c.moe_ffn, rows_e = w13 ? 2 * c.moe_ffn : c.latent;
  const int chunk = 128;   // j values (w13) or latent outputs (w2) per block
  if (!moe_tma_fits(c)) return false;
  const bool rb1 = gs == 32;
  const int GM = rb1 ? 0 : gs == K ? 1 : 2;
  const int8_t* wq = wq0 + (size_t)io.e0 * rows_e * K;
  const float* wsc = wsc0 + (size_t)io.e0 * rows_e * (K / gs);
  MoeTmaArgs a;
  memset(&a, 0, sizeof(a));
  const CUtensorMap* mq = tmap(s, wq, K, io.ne * rows_e, 128, 128);
  const CUtensorMap* ms = rb1 ? tmap(s, wsc, K / 32, io.ne * rows_e, 4, 128) : nullptr;
  if (!mq || (rb1 && !ms)) return false;
  a.wq = *mq;
  if (rb1) a.wsc = *ms;
  a.ws = wsc; a.list = io.list; a.tiles = io.tiles; a.ntiles = io.ntiles;
  a.xq = w13 ? io.latq : io.hq; a.xs = w13 ? io.lats : io.hs;
  a.hq = io.hq; a.hs = io.hs; a.h2 = io.h2; a.err = s->d_err;
  a.K = K; a.gs = gs; a.rows_e = rows_e; a.ffn = c.moe_ffn; a.latent = c.latent; a.topk = io.topk;
  const dim3 grid((w13 ? c.moe_ffn : c.latent) / chunk, tmax);
  if (s->prof) {
    // algorithmic bytes with every expert touched (R >= 4 E / top_k makes
    // an untouched expert unlikely): int8 weights + their scales
    const double rows = (double)io.ne * rows_e;
    s->prof_moe_bytes.push_back(rows * K + rows * (K / gs) * 4.0);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, s->st);
    s->prof_moe_ev.push_back(e0);
    s->prof_moe_ev.push_back(e1);
  }
#define LZ_MOE(W, RB, G) \
  launch(s, moe_tma_kernel<W, RB, G>, grid, dim3((MoeTma<W, RB>::CW + 1) * 32), MoeTma<W, RB>::smem(K), a)
  if (w13) {
    if (GM == 0) LZ_MOE(true, true, 0);
    else if (GM == 1) LZ_MOE(true, false, 1);
    else LZ_MOE(true, false, 2);
  } else {
    if (GM == 0) LZ_MOE(false, true, 0);
    else if (GM == 1) LZ_MOE(false, false, 1);
    else LZ_MOE(false, false, 2);
  }
#undef LZ_MOE
  if (s->prof) cudaEventRecord(s->prof_moe_ev.back(), s->st);
  return true;
}

// R > 8 token rows with K (and K2) % 128 == 0: the TMA-staged tensor-core
// GEMM.  Tiles: 32-row token tiles while the grid stays within ~4 blocks
// per SM, 64-row ones above; 64-output tiles for the wide lm_head at
// R <= 32.  False when the shape does not fit (the caller then launches
// the warp-tile kernel).
bool gemm_tma(LZRunState* s, const QW& w, const int8_t* xq, const float* xs, int R, float* y, int ldy, int mode,
              const QW* w2, const int8_t* xq2, const float* xs2) {
  if (w.in % 128 || (w2 && w2->in % 128)) return false;
  const bool rb1 = w.gs == 32;
  const int GM = rb1 ? 0 : (w.gs == w.in && (!w2 || w2->gs == w2->in)) ? 1 : 2;
  int MT = 1, NT = 1;
  if (R <= 32) NT = w.out >= 8192 ? 2 : 1;
  else MT = (long)((w.out + 31) / 32) * ((R + 31) / 32) <= 4L * s->n_sm ? 1 : 2;
  const int BM = 32 * MT, BN = 32 * NT;
  GemmTmaArgs a;
  memset(&a, 0, sizeof(a));
  const CUtensorMap* m[8] = {tmap(s, xq, w.in, R, 128, BM), tmap(s, xs, w.in / 32, R, 4, BM),
                             tmap(s, w.q, w.in, w.out, 128, BN), rb1 ? tmap(s, w.s, w.in / 32, w.out, 4, BN) : nullptr,
                             nullptr, nullptr, nullptr, nullptr};
  if (w2) {
    m[4] = tmap(s, xq2, w2->in, R, 128, BM);
    m[5] = tmap(s, xs2, w2->in / 32, R, 4, BM);
    m[6] = tmap(s, w2->q, w2->in, w.out, 128, BN);
    m[7] = rb1 ? tmap(s, w2->s, w2->in / 32, w.out, 4, BN) : nullptr;
  }
  for (int i = 0; i < (w2 ? 8 : 4); i++)
    if (!m[i] && (rb1 || (i & 3) != 3)) return false;
  a.a = *m[0]; a.x = *m[1]; a.b = *m[2];
  if (rb1) a.w = *m[3];
  if (w2) {
    a.a2 = *m[4]; a.x2 = *m[5]; a.b2 = *m[6];
    if (rb1) a.w2 = *m[7];
  }
  a.ws = w.s; a.ws2 = w2 ? w2->s : nullptr; a.W = w.q; a.W2 = w2 ? w2->q : nullptr;
  a.y = y; a.err = s->d_err;
  a.N = w.out; a.K = w.in; a.gs = w.gs; a.K2 = w2 ? w2->in : 0; a.gs2 = w2 ? w2->gs : 32;
  a.R = R; a.ldy = ldy; a.mode = mode; a.dual = w2 ? 1 : 0;
  const int v = MT * 10 + NT;
  if (GM == 0) {
    if (v == 11) tma_launch<1, 1, true, 0>(s, a);
    else if (v == 12) tma_launch<1, 2, true, 0>(s, a);
    else tma_launch<2, 1, true, 0>(s, a);
  } else if (GM == 1) {
    if (v == 11) tma_launch<1, 1, false, 1>(s, a);
    else if (v == 12) tma_launch<1, 2, false, 1>(s, a);
    else tma_launch<2, 1, false, 1>(s, a);
  } else {
    if (v == 11) tma_launch<1, 1, false, 2>(s, a);
    else if (v == 12) tma_launch<1, 2, false, 2>(s, a);
    else tma_launch<2, 1, false, 2>(s, a);
  }
  return true;
}

// R > 8 token rows with K (and K2) % 128 == 0 on the tcgen05 kernel: 128
// weight rows x 16 token rows per CTA.  False when a map cannot be built.
bool gemm_umma(LZRunState* s, const QW& w, const int8_t* xq, const float* xs, int R, float* y, int ldy, int mode,
               const QW* w2, const int8_t* xq2, const float* xs2) {
  if (w.in % 128 || (w2 && w2->in % 128)) return false;
  const bool rb1 = w.gs == 32;
  const int GM = rb1 ? 0 : (w.gs == w.in && (!w2 || w2->gs == w2->in)) ? 1 : 2;
  constexpr int NT = 16;
  GemmTmaArgs a;
  memset(&a, 0, sizeof(a));
  const CUtensorMap* m[8] = {tmap(s, xq, w.in, R, 128, NT), tmap(s, xs, w.in / 32, R, 4, NT),
                             tmap(s, w.q, w.in, w.out, 128, kUmmaM),
                             rb1 ? tmap(s, w.s, w.in / 32, w.out, 4, kUmmaM) : nullptr,
                             nullptr, nullptr, nullptr, nullptr};
  if (w2) {
    m[4] = tmap(s, xq2, w2->in, R, 128, NT);
    m[5] = tmap(s, xs2, w2->in / 32, R, 4, NT);
    m[6] = tmap(s, w2->q, w2->in, w.out, 128, kUmmaM);
    m[7] = rb1 ? tmap(s, w2->s, w2->in / 32, w.out, 4, kUmmaM) : nullptr;
  }
  for (int i = 0; i < (w2 ? 8 : 4); i++)
    if (!m[i] && (rb1 || (i & 3) != 3)) return false;
  a.a = *m[0]; a.x = *m[1]; a.b = *m[2];
  if (rb1) a.w = *m[3];
  if (w2) {
    a.a2 = *m[4]; a.x2 = *m[5]; a.b2 = *m[6];
    if (rb1) a.w2 = *m[7];
  }
  a.ws = w.s; a.ws2 = w2 ? w2->s : nullptr; a.W = w.q; a.W2 = w2 ? w2->q : nullptr;
  a.y = y; a.err = s->d_err;
  a.N = w.out; a.K = w.in; a.gs = w.gs; a.K2 = w2 ? w2->in : 0; a.gs2 = w2 ? w2->gs : 32;
  a.R = R; a.ldy = ldy; a.mode = mode; a.dual = w2 ? 1 : 0;
  const dim3 grid((w.out + kUmmaM - 1) / kUmmaM, (R + NT - 1) / NT);
  if (GM == 0) launch(s, gemm_q8_umma_kernel<NT, 0>, grid, dim3(kUmmaThreads), UmmaTile<NT, true>::smem(), a);
  else if (GM == 1) launch(s, gemm_q8_umma_kernel<NT, 1>, grid, dim3(kUmmaThreads), UmmaTile<NT, false>::smem(), a);
  else launch(s, gemm_q8_umma_kernel<NT, 2>, grid, dim3(kUmmaThreads), UmmaTile<NT, false>::smem(), a);
  return true;
}

// y (R x N, ld ldy) = [y +] W x (+ W2 x2).  With `nin`, x is produced here
// from the float rows nin->x by RMSNorm + quantisation: inside the GEMV
// (every block, from shared memory) for R <= kPrologueRows, else by one
// rmsnorm_quant grid into xq/xs first.
void gemv(LZRunState* s, const QW& w, int8_t* xq, float* xs, int R, float* y, int ldy,
          int mode = 0, const QW* w2 = nullptr, const int8_t* xq2 = nullptr, const float* xs2 = nullptr,
          const InNorm* nin = nullptr, const GemvFuse* fz = nullptr) {
  GemvArgs a{w.q, w.s, w.out, w.in, w.gs, xq, xs, R, y, ldy, mode,
             w2 ? w2->q : nullptr, w2 ? w2->s : nullptr, w2 ? w2->in : 0, w2 ? w2->gs : 32, xq2, xs2,
             nullptr, nullptr, s->m->c.eps, nullptr, nullptr, {}};
  const bool prologue = nin && R <= kPrologueRows;
  if (prologue) {
    a.nx = nin->x; a.nw = nin->w; a.nout = nin->out; a.namax = nin->amax;
    // the fused greedy tail: the slots were cleared by the round's setup kernel
    if (fz) {
      a.fz = *fz;
      a.namax = nullptr;
    }
  } else if (nin) {
    rmsnorm_quant(s, nin->x, w.in, nin->w, w.in, R, nin->out, w.in, xq, xs, nin->amax);
  }
  const int nsb = std::max(w.in, w2 ? w2->in : 0) / 32;
  if (s->prof) {
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, s->st);
    s->prof_ev.push_back(e0);
    s->prof_ev.push_back(e1);
    // algorithmic bytes: weights + weight scales + activations + outputs
    auto bytes = [R](const QW& q) {
      return (double)q.out * q.in + (double)q.out * (q.in / q.gs) * 4.0 + (double)R * q.in +
             (double)R * (q.in / 32) * 4.0;
    };
    double b = bytes(w) + (w2 ? bytes(*w2) : 0.0) + (double)R * w.out * 4.0 * (mode ? 2.0 : 1.0);
    s->prof_bytes.push_back(b);
  }
  const bool rb1 = w.gs == 32;
  if (R > kPrologueRows && (!w2 || (w2->gs == 32) == rb1) && s->umma &&
      gemm_umma(s, w, xq, xs, R, y, ldy, mode, w2, xq2, xs2)) {
    // launched
  } else if (R > kPrologueRows && (!w2 || (w2->gs == 32) == rb1) &&
             gemm_tma(s, w, xq, xs, R, y, ldy, mode, w2, xq2, xs2)) {
    // launched
  } else if (R > kPrologueRows && (!w2 || (w2->gs == 32) == rb1)) {
    // tensor-core warp tiles of 16 MT token rows x 8 NT outputs (measured
    // best: 32 x 16 for wide outputs, 32 x 8 for narrow ones, 16-row tiles
    // when R <= 16)
    const int MT = R > 16 ? 2 : 1, NT = w.out >= 2048 ? 2 : 1;
    const dim3 grid((w.out + 32 * NT - 1) / (32 * NT), (R + 16 * MT - 1) / (16 * MT));
#define LZ_GEMM(mt, nt)                                                                   \
  if (rb1) launch(s, gemm_q8_warp_kernel<mt, nt, true>, grid, dim3(128), 0, a);           \
  else launch(s, gemm_q8_warp_kernel<mt, nt, false>, grid, dim3(128), 0, a);
    if (MT == 1 && NT == 1) { LZ_GEMM(1, 1) }
    else if (MT == 1) { LZ_GEMM(1, 2) }
    else if (NT == 1) { LZ_GEMM(2, 1) }
    else { LZ_GEMM(2, 2) }
#undef LZ_GEMM
  } else if (prologue) {
    if (nsb <= 32) gemv_launch_rb<1, kGemvProWarps, true>(s, a);
    else gemv_launch_rb<2, kGemvProWarps, true>(s, a);
  } else if (w2 || R > kGemvRB) {
    if (nsb <= 32) gemv_launch<1, kGemvWarps, kGemvRB, false, true>(s, a);
    else if (nsb <= 64) gemv_launch<2, kGemvWarps, kGemvRB, false, true>(s, a);
    else gemv_launch<4, kGemvWarps, kGemvRB, false, true>(s, a);
  } else {
    if (nsb <= 32) gemv_launch_rb<1, kGemvWarps, false>(s, a);
    else if (nsb <= 64) gemv_launch_rb<2, kGemvWarps, false>(s, a);
    else gemv_launch_rb<4, kGemvWarps, false>(s, a);
  }
  if (s->prof) cudaEventRecord(s->prof_ev.back(), s->st);
}

void rmsnorm_quant(LZRunState* s, const float* x, int ldx, const float* w, int n, int R, float* out,
                   int ldo, int8_t* xq, float* xs, unsigned long long* amax_clear) {
  // the row, its weights, and the squares of the split sum of squares
  launch(s, rmsnorm_quant_kernel, dim3(R), dim3(256), (3 * n + 16) * sizeof(float), x, ldx, w, n, s->m->c.eps, out, ldo, xq, xs,
                                                                 amax_clear);
}

void argmax(LZRunState* s, const float* logits, int R, int p1_mode) {
  const int V = s->m->c.vocab;
  launch(s, argmax_kernel, dim3((V + kArgmaxChunk - 1) / kArgmaxChunk, R), dim3(256), 0, logits, V, p1_mode, s->vmax);
}

// The routed experts of io's pairs (src/forward_moe.c:55-206): pairs
// bucketed by expert into tiles of 8 pairs (TMA-staged kernels) or 16
// (warp-tile kernels), w1/w3 with SiLU x up and the per-32 quantisation,
// then w2 into io.h2 (one latent row per pair).
void grouped_experts(LZRunState* s, const DLayer& L, const MoeIO& io) {
  const Cfg& c = s->m->c;
  const int trows = moe_tma_fits(c) ? kMoeTileRows : 16;
  const int tmax = io.P / trows + std::min(io.ne, io.P) + 1;
  launch(s, moe_group_kernel, dim3(1), dim3(1024), 0, io.pair_e, io.P, io.ne, io.list, io.tiles, io.ntiles, trows);
  const int8_t* w13q = L.w13q + (size_t)io.e0 * 2 * c.moe_ffn * c.latent;
  const float* w13s = L.w13s + (size_t)io.e0 * 2 * c.moe_ffn * (c.latent / L.w13_gs);
  const int8_t* w2q = L.w2q + (size_t)io.e0 * c.latent * c.moe_ffn;
  const float* w2s = L.w2s + (size_t)io.e0 * c.latent * (c.moe_ffn / L.w2_gs);
  if (moe_tma(s, true, L.w13q, L.w13s, L.w13_gs, tmax, io)) {
    // launched
  } else if (L.w13_gs == 32)
    launch(s, moe_w13_group_kernel<true>, dim3((c.moe_ffn + 127) / 128, tmax), dim3(128), 0, w13q, w13s, c.moe_ffn,
           c.latent, L.w13_gs, io.list, io.tiles, io.ntiles, io.topk, io.latq, io.lats, io.hq, io.hs);
  else
    launch(s, moe_w13_group_kernel<false>, dim3((c.moe_ffn + 127) / 128, tmax), dim3(128), 0, w13q, w13s, c.moe_ffn,
           c.latent, L.w13_gs, io.list, io.tiles, io.ntiles, io.topk, io.latq, io.lats, io.hq, io.hs);
  if (moe_tma(s, false, L.w2q, L.w2s, L.w2_gs, tmax, io)) {
    // launched
  } else if (L.w2_gs == 32)
    launch(s, moe_w2_group_kernel<true>, dim3((c.latent + 63) / 64, tmax), dim3(128), 0, w2q, w2s, c.moe_ffn,
           c.latent, L.w2_gs, io.list, io.tiles, io.ntiles, io.hq, io.hs, io.h2);
  else
    launch(s, moe_w2_group_kernel<false>, dim3((c.latent + 63) / 64, tmax), dim3(128), 0, w2q, w2s, c.moe_ffn,
           c.latent, L.w2_gs, io.list, io.tiles, io.ntiles, io.hq, io.hs, io.h2);
}

// One exchange of equal-size per-peer blocks with every other rank (NCCL
// send/recv in one group, on the state's stream).
void ep_exchange(LZRunState* s, const void* send, void* recv, size_t bytes) {
  const NcclApi* n = nccl_api();
  EpCtx& E = s->ep;
  if (!n || !E.comm) {
    E.failed = true;
    return;
  }
  bool ok = n->group_start() == ncclSuccess;
  for (int p = 0; p < E.world && ok; p++) {
    if (p == E.rank) continue;
    ok = n->send(static_cast<const uint8_t*>(send) + (size_t)p * bytes, bytes, ncclUint8, p, E.comm, s->st) ==
             ncclSuccess &&
         n->recv(static_cast<uint8_t*>(recv) + (size_t)p * bytes, bytes, ncclUint8, p, E.comm, s->st) == ncclSuccess;
  }
  if (n->group_end() != ncclSuccess || !ok) E.failed = true;
}

// Expert-parallel MoE of one layer (lz98_ep.cuh): pack the pairs by owner,
// exchange, the owned experts over every rank's pairs, return the rows,
// combine in selection order.
void moe_ep(LZRunState* s, const DLayer& L, int R) {
  const Cfg& c = s->m->c;
  EpCtx& E = s->ep;
  const int P = R * c.topk;
  const EpBuf b = E.buf;
  launch(s, ep_pack_kernel, dim3(1), dim3(1024), 0, s->pair_e, P, c.topk, E.epr, s->latq, s->lats, b, E.pair_dest,
         E.pair_slot);
  ep_exchange(s, b.send, b.recv, b.buf_bytes);
  launch(s, ep_unpack_kernel, dim3(1), dim3(1024), 0, b, E.latq, E.lats, E.expert, E.src, E.slot, E.total);
  const MoeIO io{E.expert, b.world * b.cap, 1, E.epr, E.e0, E.list, E.tiles, E.ntiles, E.latq, E.lats, E.hq, E.hs,
                 E.h2};
  grouped_experts(s, L, io);
  launch(s, ep_reply_kernel, dim3(b.world * b.cap), dim3(128), 0, E.h2, E.src, E.slot, E.total, c.latent, b.cap,
         b.rank, E.sendback, E.recvback);
  ep_exchange(s, E.sendback, E.recvback, (size_t)b.cap * c.latent * sizeof(float));
  launch(s, ep_combine_kernel, dim3(R), dim3(256), 0, s->pair_e, s->pair_w, E.pair_dest, E.pair_slot, c.topk,
         E.recvback, b.cap, c.latent, s->yq, s->ys);
}

// Body forward of R rows (src/forward.c:1210-1617): embed, per layer
// pre-norm -> KDA -> residual -> post-norm -> latent MoE -> residual, then
// final norm (hidden capture) and the tied lm_head over every row.
void body_forward(LZRunState* s, int R, int nseq, int adv, bool want_logits, const GemvFuse* fz = nullptr) {
  const LZModel* m = s->m;
  const Cfg& c = m->c;
  const int d = c.d, kdim = c.key_dim, vdim = c.val_dim;
  launch(s, embed_kernel, dim3(R), dim3(256), 0, m->embed.q, m->embed.s, m->embed.gs, d, s->tok, s->x);
  for (int l = 0; l < c.nl; l++) {
    const DLayer& L = m->L[l];
    const InNorm in_ln{s->x, L.in_ln, nullptr, nullptr};
    gemv(s, L.inproj, s->xq, s->xs, R, s->inproj, m->n_in, 0, nullptr, nullptr, nullptr, &in_ln);
    KdaArgs ka{s->inproj, m->n_in, kdim, m->off_g, m->off_fa, m->off_b, c.rank, L.conv_w,
               s->conv + (size_t)l * c.conv_dim * 3, s->conv_seq, s->conv_slot, L.fb.q, L.fb.s, L.fb.gs, L.a_log,
               L.dt_bias, c.lb, s->seqs, s->hi, s->lo, s->sc, s->q_seq, s->q_slot,
               (int)((size_t)l * c.nv * c.kd * c.vd), s->depth, adv, s->ssm_scale, L.o_norm, c.eps, vdim, s->oq,
               s->os};
    // few (head, sequence) pairs (batch 1): each head as a cluster of two
    // 16-warp CTAs, one per value group; otherwise one 8-warp CTA per head,
    // 4 per SM
    if (2 * c.nv * nseq <= s->n_sm)
      launch(s, kda_recur_split_kernel<2 * kRecurThreads>, dim3(2 * c.nv, nseq), dim3(2 * kRecurThreads), 0, ka);
    else
      launch(s, kda_recur_kernel<kRecurThreads>, dim3(c.nv, nseq), dim3(kRecurThreads), 0, ka);
    gemv(s, L.o, s->oq, s->os, R, s->x, d, 1);
    const InNorm post{s->x, L.post_ln, nullptr, nullptr};
    gemv(s, L.moein, s->xq, s->xs, R, s->moein, m->n_moe, 0, nullptr, nullptr, nullptr, &post);
    const int P = R * c.topk;
    if (R <= kPrologueRows && !s->ep.comm) {
      // few rows: router fused into the per-pair w1/w3 kernel, then w2 with
      // the last-block combine
      // latent <= 512: 16 lanes per weight row, 64 FFN outputs per block
      // (one wave of blocks at batch 1); else 32 lanes, 32 outputs
      if (c.latent <= 512 && c.moe_ffn % 64 == 0)
        launch(s, moe_route_w13_kernel<16>, dim3(c.moe_ffn / 64, P), dim3(256), 0, s->moein, m->n_moe,
               m->off_router, m->off_down, L.router_bias, c.ne, c.topk, L.w13q, L.w13s, c.moe_ffn, c.latent,
               L.w13_gs, s->pair_e, s->pair_w, s->hq, s->hs, m->off_shg, m->off_shu, c.shared_w, s->shq, s->shs);
      else
        launch(s, moe_route_w13_kernel<32>, dim3(c.moe_ffn / 32, P), dim3(256), 0, s->moein, m->n_moe,
               m->off_router, m->off_down, L.router_bias, c.ne, c.topk, L.w13q, L.w13s, c.moe_ffn, c.latent,
               L.w13_gs, s->pair_e, s->pair_w, s->hq, s->hs, m->off_shg, m->off_shu, c.shared_w, s->shq, s->shs);
      launch(s, moe_w2_kernel, dim3((c.latent + 8 * kW2Rows - 1) / (8 * kW2Rows), P), dim3(256), 0, L.w2q, L.w2s,
             c.moe_ffn, c.latent,
             L.w2_gs, s->pair_e, s->pair_w, c.topk, s->hq, s->hs, s->h2, s->row_counter, s->yq, s->ys);
    } else {
      launch(s, moe_route_kernel, dim3(R), dim3(512), 0, s->moein, m->n_moe, m->off_router, m->off_down,
             L.router_bias, c.ne, c.topk, c.latent, s->pair_e, s->pair_w, s->latq, s->lats, m->off_shg, m->off_shu,
             c.shared_w, s->shq, s->shs);
      if (s->ep.comm) {
        moe_ep(s, L, R);
      } else {
        const MoeIO io{s->pair_e, P, c.topk, c.ne, 0, s->glist, s->gtiles, s->gntiles, s->latq, s->lats,
                       s->hq, s->hs, s->h2};
        grouped_experts(s, L, io);
        launch(s, moe_combine_kernel, dim3(R), dim3(256), 0, s->pair_e, s->pair_w, c.topk, s->h2, c.latent, s->yq,
               s->ys);
      }
    }
    if (c.shared_w) gemv(s, L.up, s->yq, s->ys, R, s->x, d, 1, &L.sh_down, s->shq, s->shs);
    else gemv(s, L.up, s->yq, s->ys, R, s->x, d, 1);
  }
  // final norm: hidden capture, then the tied lm_head
  if (want_logits) {
    const InNorm fin{s->x, m->final_norm, s->hidden, s->vmax};
    gemv(s, m->embed, s->xq, s->xs, R, s->logits, c.vocab, 0, nullptr, nullptr, nullptr, &fin, fz);
  } else {
    rmsnorm_quant(s, s->x, d, m->final_norm, d, R, s->hidden, d, s->xq, s->xs, s->vmax);
  }
}

// MTP block over R rows (src/forward_mtp.c:32-144, 561-624): fc front,
// input norm, q|k|v projection, cache write; when `full`, the gated
// attention, o_proj, dense SwiGLU FFN, final norm into chain_out and the
// tied lm_head into s->logits.
void mtp_forward(LZRunState* s, int R, const int* tok, const float* hid, const int* hid_idx,
                 const MtpRow* rows, bool full, float* chain_out, const GemvFuse* fz = nullptr) {
  const LZModel* m = s->m;
  const Cfg& c = m->c;
  const DMtp& M = m->mtp;
  const int d = c.d;
  launch(s, mtp_front_kernel, dim3(R), dim3(256), (4 * d + 32) * sizeof(float), m->embed.q, m->embed.s, m->embed.gs, d, tok,
                                                             hid, hid_idx, M.pre_e, M.pre_h, c.eps, s->xq,
                                                             s->xs);
  gemv(s, M.fc, s->xq, s->xs, R, s->mtpx, d);
  const InNorm in_ln{s->mtpx, M.in_ln, nullptr, nullptr};
  gemv(s, M.qkv, s->xq, s->xs, R, s->qkv, m->n_qkv, 0, nullptr, nullptr, nullptr, &in_ln);
  launch(s, mtp_kv_write_kernel, dim3(c.nkv, R), dim3(64), 0, s->qkv, m->n_qkv, m->off_mk, m->off_mv, rows, M.k_norm,
                                                        c.eps, c.hd, c.rot, c.kv_dim, s->rope, s->kq, s->ks,
                                                        s->vq, s->vs, s->cache_seq);
  if (!full) return;
  const size_t smem = (size_t)s->seq_len * sizeof(float);
  launch(s, mtp_attn_kernel, dim3(c.nh, R), dim3(kAttnThreads), smem, 
      s->qkv, m->n_qkv, c.q_dim, rows, M.q_norm, c.eps, c.hd, c.rot, c.kv_dim, c.nh / c.nkv, s->rope,
      s->attn_scale, s->kq, s->ks, s->vq, s->vs, s->cache_seq, s->aq, s->as);
  gemv(s, M.o, s->aq, s->as, R, s->mtpx, d, 1);
  const InNorm post{s->mtpx, M.post_ln, nullptr, nullptr};
  gemv(s, M.gu, s->xq, s->xs, R, s->inproj, 2 * c.mtp_ffn, 0, nullptr, nullptr, nullptr, &post);
  launch(s, swiglu_quant_kernel, dim3(R), dim3(256), 0, s->inproj, 2 * c.mtp_ffn, 0, c.mtp_ffn, c.mtp_ffn, s->shq, s->shs);
  gemv(s, M.down, s->shq, s->shs, R, s->mtpx, d, 1);
  const InNorm fin{s->mtpx, M.norm, chain_out, s->vmax};
  gemv(s, m->embed, s->xq, s->xs, R, s->logits, c.vocab, 0, nullptr, nullptr, nullptr, &fin, fz);
}

__global__ void set_rows_kernel(MtpRow* rows, int n, int seq, int pos0, int seq_len) {
  pdl_trigger();
  pdl_wait();
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) rows[i] = MtpRow{seq, pos0 + i, pos0 + i >= 0 && pos0 + i < seq_len};
}

// Rows whose MTP position would fall outside the cache are marked
// inactive (no cache write, no attention): the memory stays in bounds and
// the host's budget check (max_pos) keeps such rounds from being asked for.
// Also clears the rows' arg-max slots, which a fused lm_head folds into.
__global__ void draft_setup_kernel(const SeqRound* sr, int nseq, int i, int seq_len, int* tok, MtpRow* rows,
                                   unsigned long long* amax) {
  pdl_trigger();
  pdl_wait();
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nseq) return;
  amax[b] = 0ull;
  tok[b] = i == 0 ? sr[b].anchor : sr[b].draft[i - 1];
  const int pos = sr[b].mtp_pos + i;
  rows[b] = MtpRow{b, pos, pos >= 0 && pos < seq_len};
}

__global__ void draft_store_kernel(SeqRound* sr, int nseq, int i, int k, const unsigned long long* amax) {
  pdl_trigger();
  pdl_wait();
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nseq) return;
  sr[b].draft[i] = argmax_index(amax[b]);
  sr[b].k = k;
}

// Also clears the verify rows' arg-max slots, which a fused lm_head folds into.
__global__ void verify_setup_kernel(const SeqRound* sr, int nseq, int k, int* tok, KdaSeq* seqs,
                                    unsigned long long* amax) {
  pdl_trigger();
  pdl_wait();
  int b = blockIdx.x;
  if (b >= nseq) return;
  if (threadIdx.x == 0) seqs[b] = KdaSeq{b * (k + 1), k + 1, sr[b].ssm_slot, b};
  for (int j = threadIdx.x; j <= k; j += blockDim.x) {
    tok[b * (k + 1) + j] = j == 0 ? sr[b].anchor : sr[b].draft[j - 1];
    amax[b * (k + 1) + j] = 0ull;
  }
}

int upload_seqs(LZRunState* s, const std::vector<KdaSeq>& v) {
  CK(cudaMemcpyAsync(s->seqs, v.data(), v.size() * sizeof(KdaSeq), cudaMemcpyHostToDevice, s->st));
  return 0;
}

// Debug timing marks of a round: 0 before drafting, 1 before the verify, 2
// after the acceptance, 3 after the catch-up.
void dbg_mark(LZRunState* s, int i) {
  // external records become event nodes of a captured round graph
  if (s->dbg_timing) cudaEventRecordWithFlags(s->dbg_ev[i], s->st, cudaEventRecordExternal);
}

// The verify half of a greedy round with drafts sr[b].draft[0..k) and
// sr[b].k == k: the (k+1)-row verify, acceptance, ring, chain reseed and
// catch-up.
void verify_greedy(LZRunState* s, int k) {
  const Cfg& c = s->m->c;
  const int B = s->B, R = B * (k + 1);
  launch(s, verify_setup_kernel, dim3(B), dim3(32), 0, s->sr, B, k, s->tok, s->seqs, s->vmax);
  if (R <= kPrologueRows) {
    // logits to acceptance in the lm_head's own launch: arg-max folded into
    // its reductions, the acceptance by its last block
    const GemvFuse fz{s->vmax, 0, s->sr, B, k, s->hidden, c.d, s->chain, s->depth, s->seq_len, s->crows,
                      s->catch_tok, s->catch_hidx, s->accept_counter};
    body_forward(s, R, B, 1, true, &fz);
  } else {
    body_forward(s, R, B, 1, true);
    argmax(s, s->logits, R, 0);
    launch(s, spec_accept_greedy_kernel, dim3(B), dim3(256), 0, s->sr, B, k, s->vmax, s->hidden, c.d, s->chain,
           s->depth, s->seq_len, s->crows, s->catch_tok, s->catch_hidx);
  }
  dbg_mark(s, 2);
  if (k > 1)
    mtp_forward(s, B * (k - 1), s->catch_tok, s->hidden, s->catch_hidx, s->crows, false, nullptr);
  dbg_mark(s, 3);
}

// The verify half of a temperature round (drafts and their q rows in place).
void verify_temp(LZRunState* s, int k) {
  const Cfg& c = s->m->c;
  const int B = s->B, V = c.vocab, R = B * (k + 1);
  launch(s, verify_setup_kernel, dim3(B), dim3(32), 0, s->sr, B, k, s->tok, s->seqs, s->vmax);
  body_forward(s, R, B, 1, true);
  launch(s, temp_target_kernel, dim3(R), dim3(kSampThreads), kSampSmem, s->logits, V, s->sr, k, s->pbuf,
         s->sortbuf, s->npow2);
  launch(s, temp_accept_kernel, dim3(B), dim3(kSampThreads), kSampSmem, s->sr, k, s->kmax, s->pbuf, s->qbuf, V,
         s->hidden, c.d, s->chain, s->depth, s->seq_len, s->crows, s->catch_tok, s->catch_hidx);
  dbg_mark(s, 2);
  if (k > 1)
    mtp_forward(s, B * (k - 1), s->catch_tok, s->hidden, s->catch_hidx, s->crows, false, nullptr);
  dbg_mark(s, 3);
}

// One greedy round of every sequence, all on the device.
void round_greedy(LZRunState* s, int k) {
  const int B = s->B;
  const int tb = (B + 127) / 128;
  dbg_mark(s, 0);
  for (int i = 0; i < k; i++) {
    launch(s, draft_setup_kernel, dim3(tb), dim3(128), 0, s->sr, B, i, s->seq_len, s->tok, s->mrows, s->vmax);
    if (B <= kPrologueRows) {
      // the draft arg-max folded into the lm_head's reductions
      const GemvFuse fz{s->vmax, 1, nullptr, 0, 0, nullptr, 0, nullptr, 0, 0, nullptr, nullptr, nullptr, nullptr};
      mtp_forward(s, B, s->tok, s->chain, nullptr, s->mrows, true, s->chain, &fz);
    } else {
      mtp_forward(s, B, s->tok, s->chain, nullptr, s->mrows, true, s->chain);
      argmax(s, s->logits, B, 1);
    }
    launch(s, draft_store_kernel, dim3(tb), dim3(128), 0, s->sr, B, i, k, s->vmax);
  }
  dbg_mark(s, 1);
  verify_greedy(s, k);
}

// One temperature round of every sequence (src/generate.c:1234-1377), all
// on the device: k draft steps sampling q, the (k+1)-row verify, target
// distributions, coupled acceptance, then the greedy round's ring,
// chain and catch-up steps.
void round_temp(LZRunState* s, int k) {
  const LZModel* m = s->m;
  const Cfg& c = m->c;
  const int B = s->B, V = c.vocab;
  const int tb = (B + 127) / 128;
  dbg_mark(s, 0);
  for (int i = 0; i < k; i++) {
    launch(s, draft_setup_kernel, dim3(tb), dim3(128), 0, s->sr, B, i, s->seq_len, s->tok, s->mrows, s->vmax);
    mtp_forward(s, B, s->tok, s->chain, nullptr, s->mrows, true, s->chain);
    launch(s, temp_draft_kernel, dim3(B), dim3(kSampThreads), kSampSmem, s->logits, V, s->sr, i, k, s->kmax,
           s->qbuf);
  }
  dbg_mark(s, 1);
  verify_temp(s, k);
}

// 0: every sequence greedy, 1: every sequence in temperature mode, -1: mixed.
int round_mode(const LZRunState* s) {
  int t = 0;
  for (char v : s->seq_temp) t += v != 0;
  return t == 0 ? 0 : (t == (int)s->seq_temp.size() ? 1 : -1);
}

void round_any(LZRunState* s, int k) {
  if (round_mode(s) == 1) round_temp(s, k);
  else round_greedy(s, k);
}

// Drafting of sequence 0 with the early stop of p_min (src/generate.c:
// 741-762 greedy, 1258-1280 temperature): step by step, each step's
// confidence read back - lz_argmax_p1's probability of the greedy draft,
// q(x) of the sampled one - and the first step below p_min not recorded.
// Returns k_eff, or -1 on a CUDA failure.
int draft_pmin(LZRunState* s, int k, bool temp, float p_min) {
  const Cfg& c = s->m->c;
  int k_eff = 0;
  dbg_mark(s, 0);
  for (int i = 0; i < k; i++) {
    launch(s, draft_setup_kernel, dim3(1), dim3(128), 0, s->sr, 1, i, s->seq_len, s->tok, s->mrows, s->vmax);
    mtp_forward(s, 1, s->tok, s->chain, nullptr, s->mrows, true, s->chain);
    float conf = 0.0f;
    if (temp) {
      launch(s, temp_draft_kernel, dim3(1), dim3(kSampThreads), kSampSmem, s->logits, c.vocab, s->sr, i, k, s->kmax,
             s->qbuf);
      if (!sr_down(s)) return -1;
      const int x = s->h_sr[0].draft[i];
      if (cudaMemcpyAsync(&conf, s->qbuf + (size_t)i * c.vocab + x, 4, cudaMemcpyDeviceToHost, s->st) != cudaSuccess)
        return -1;
    } else {
      launch(s, argmax_p1_kernel, dim3(1), dim3(kSampThreads), kSampSmem, s->logits, c.vocab, s->sr, i, k,
             reinterpret_cast<int*>(s->sortbuf), s->pconf);
      if (cudaMemcpyAsync(&conf, s->pconf, 4, cudaMemcpyDeviceToHost, s->st) != cudaSuccess) return -1;
    }
    if (!sync_ok(s)) return -1;
    if (conf < p_min) break;
    k_eff = i + 1;
  }
  return k_eff;
}

// A round of sequence 0 with p_min / n_min (eager): drafting as above; a
// draft shorter than n_min is discarded (returns 0: no verify, positions
// unchanged, src/generate.c:765-791), else the verify half runs at k_eff.
// Returns -1 on a CUDA failure, else 0 (discarded) or 1.
int round_pmin(LZRunState* s, int k, bool temp, float p_min, int n_min, int* k_eff) {
  *k_eff = draft_pmin(s, k, temp, p_min);
  if (*k_eff < 0) return -1;
  if (*k_eff < n_min) return 0;   // k_eff == 0 with n_min == 0 still verifies the anchor row
  if (!sr_down(s)) return -1;
  s->h_sr[0].k = *k_eff;
  if (!sr_up(s)) return -1;
  dbg_mark(s, 1);
  if (temp) verify_temp(s, *k_eff);
  else verify_greedy(s, *k_eff);
  return sync_ok(s) ? 1 : -1;
}

// One token of sequence `seq` from logits row 0 by its sampler (arg-max at
// the temperature floor), on the device; the sampler state advances there.
int sample_row(LZRunState* s, int seq, int* tok) {
  const Cfg& c = s->m->c;
  launch(s, sample_row_kernel, dim3(1), dim3(kSampThreads), kSampSmem, s->logits, c.vocab, s->sr, seq, s->pbuf,
         s->sortbuf, s->npow2, s->tok_out);
  CK(cudaMemcpyAsync(tok, s->tok_out, sizeof(int), cudaMemcpyDeviceToHost, s->st));
  return sync_ok(s) ? 0 : LZ98_ERR_CUDA;
}

}  // namespace

// ============================================================ debug counters
//
// The reference's exported debug data (src/forward.c:86-124,
// src/generate.c:226): microseconds of host time in capture forwards,
// verify forwards, draft steps and catch-ups, their call counts, and the
// number of rounds that rolled the state ring back (n_accept < k_eff).
// The direct entry points time themselves; a device round is split into
// its draft / verify / catch-up parts by CUDA events when
// lz_set_debug_timing is on (off by default: the events cut the
// programmatic-launch overlap at their boundaries).
extern "C" {
long long lz_debug_us_verify = 0;
long long lz_debug_us_draft = 0;
long long lz_debug_us_capture = 0;
long long lz_debug_n_capture = 0;
long long lz_debug_us_catchup = 0;
long long lz_debug_n_catchup = 0;
long long lz_debug_n_ring_rollback = 0;
}

namespace {
struct UsTimer {
  long long* acc;
  std::chrono::steady_clock::time_point t0 = std::chrono::steady_clock::now();
  explicit UsTimer(long long* a) : acc(a) {}
  ~UsTimer() {
    *acc += std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
  }
};

// Adds the event-timed parts of the last device round of sequence 0 (when
// debug timing recorded them) and counts a rollback.
void round_debug(LZRunState* s, int n_accept, int k_eff) {
  if (n_accept < k_eff) lz_debug_n_ring_rollback++;
  if (!s->dbg_timing) return;
  float a = 0.0f, b = 0.0f, c = 0.0f;
  if (cudaEventElapsedTime(&a, s->dbg_ev[0], s->dbg_ev[1]) == cudaSuccess &&
      cudaEventElapsedTime(&b, s->dbg_ev[1], s->dbg_ev[2]) == cudaSuccess &&
      cudaEventElapsedTime(&c, s->dbg_ev[2], s->dbg_ev[3]) == cudaSuccess) {
    lz_debug_us_draft += (long long)(a * 1000.0f);
    lz_debug_us_verify += (long long)(b * 1000.0f);
    lz_debug_us_catchup += (long long)(c * 1000.0f);
  } else {
    cudaGetLastError();   // a failed timing query is not a failure of the round
  }
}
}  // namespace

extern "C" int lz_set_debug_timing(LZRunState* s, int enable) {
  if (!s) return LZ98_ERR_NULL_ARG;
  const bool on = enable != 0;
  if (on && !s->dbg_ev[0])
    for (auto& e : s->dbg_ev)
      if (cudaEventCreate(&e) != cudaSuccess) return LZ98_ERR_CUDA;
  if (on != s->dbg_timing) {
    for (auto& kv : s->graph) cudaGraphExecDestroy(kv.second);
    s->graph.clear();
  }
  s->dbg_timing = on;
  return 0;
}

// ================================================================== forwards

static float* forward_one(const LZModel* m, LZRunState* s, const int* tokens, int n, int pos0, bool capture,
                          float* hidden_out, bool all_logits) {
  const Cfg& c = m->c;
  if (!m || !s || !tokens || n < 1) return nullptr;
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= c.vocab || pos0 + i < 0 || pos0 + i >= s->seq_len) return nullptr;
  if (!sr_down(s)) return nullptr;
  const int slot = s->h_sr[0].ssm_slot;
  float* last = nullptr;
  for (int done = 0; done < n;) {
    const int R = std::min(s->Rmax, n - done);
    cudaMemcpyAsync(s->tok, tokens + done, R * sizeof(int), cudaMemcpyHostToDevice, s->st);
    upload_seqs(s, {KdaSeq{0, R, slot, 0}});
    const bool logits_here = all_logits || done + R == n;
    body_forward(s, R, 1, 0, logits_here);
    if (hidden_out)
      cudaMemcpyAsync(hidden_out + (size_t)done * c.d, s->hidden, (size_t)R * c.d * 4, cudaMemcpyDeviceToHost,
                      s->st);
    if (logits_here) {
      const int r0 = all_logits ? 0 : R - 1;
      const int nr = all_logits ? R : 1;
      cudaMemcpyAsync(s->h_logits.data() + (all_logits ? (size_t)done * c.vocab : 0),
                      s->logits + (size_t)r0 * c.vocab, (size_t)nr * c.vocab * 4, cudaMemcpyDeviceToHost,
                      s->st);
      last = s->h_logits.data();
    }
    if (capture && done + R == n)
      cudaMemcpyAsync(s->chain, s->hidden + (size_t)(R - 1) * c.d, c.d * 4, cudaMemcpyDeviceToDevice, s->st);
    done += R;
  }
  if (!sync_ok(s)) return nullptr;
  return last;
}

extern "C" float* lz_forward(const LZModel* m, LZRunState* s, int token, int pos) {
  return forward_one(m, s, &token, 1, pos, false, nullptr, false);
}

extern "C" float* lz_forward_capture(const LZModel* m, LZRunState* s, int token, int pos) {
  UsTimer t(&lz_debug_us_capture);
  lz_debug_n_capture++;
  return forward_one(m, s, &token, 1, pos, true, nullptr, false);
}

extern "C" float* lz_forward_batch_capture(const LZModel* m, LZRunState* s, const int* tokens, int n, int pos0,
                                           float* hidden_out) {
  if (!hidden_out) return nullptr;
  return forward_one(m, s, tokens, n, pos0, false, hidden_out, false);
}

extern "C" int lz_forward_verify(const LZModel* m, LZRunState* s, const int* tokens, int n, int pos0) {
  UsTimer t(&lz_debug_us_verify);
  if (!m || !s || !tokens || n < 1 || n > s->kmax + 1) return 1;
  const Cfg& c = m->c;
  for (int i = 0; i < n; i++)
    if (tokens[i] < 0 || tokens[i] >= c.vocab || pos0 + i < 0 || pos0 + i >= s->seq_len) return 1;
  if (!sr_down(s)) return 1;
  const int slot = s->h_sr[0].ssm_slot;
  cudaMemcpyAsync(s->tok, tokens, n * sizeof(int), cudaMemcpyHostToDevice, s->st);
  upload_seqs(s, {KdaSeq{0, n, slot, 0}});
  body_forward(s, n, 1, 1, true);
  cudaMemcpyAsync(s->h_logits.data(), s->logits, (size_t)n * c.vocab * 4, cudaMemcpyDeviceToHost, s->st);
  cudaMemcpyAsync(s->h_hidden.data(), s->hidden, (size_t)n * c.d * 4, cudaMemcpyDeviceToHost, s->st);
  s->h_sr[0].ssm_slot = (slot + n) % s->depth;
  return sr_up(s) && sync_ok(s) ? 0 : 1;
}

extern "C" const float* lz_state_mtp_logits(const LZRunState* s) { return s ? s->h_logits.data() : nullptr; }
extern "C" const float* lz_state_mtp_verify_hidden(const LZRunState* s) {
  return s ? s->h_hidden.data() : nullptr;
}

extern "C" float* lz_mtp_draft_step(const LZModel* m, LZRunState* s, int next_token, int pos) {
  UsTimer t(&lz_debug_us_draft);
  if (!m || !s) return nullptr;
  const Cfg& c = m->c;
  if (next_token < 0 || next_token >= c.vocab || pos < 0 || pos >= s->seq_len) return nullptr;
  cudaMemcpyAsync(s->tok, &next_token, sizeof(int), cudaMemcpyHostToDevice, s->st);
  launch(s, set_rows_kernel, dim3(1), dim3(32), 0, s->mrows, 1, 0, pos, s->seq_len);
  mtp_forward(s, 1, s->tok, s->chain, nullptr, s->mrows, true, s->chain);
  cudaMemcpyAsync(s->h_draft.data(), s->logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, s->st);
  if (!sync_ok(s)) return nullptr;
  return s->h_draft.data();
}

static int mtp_prefill_seq(LZRunState* s, int seq, const float* h_host, const float* h_dev, const int* next,
                           int n, int pos0) {
  const Cfg& c = s->m->c;
  for (int done = 0; done < n;) {
    const int R = std::min(s->Rmax, n - done);
    cudaMemcpyAsync(s->catch_tok, next + done, R * sizeof(int), cudaMemcpyHostToDevice, s->st);
    const float* hid = h_dev ? h_dev + (size_t)done * c.d : s->mtpx;
    if (h_host) {
      cudaMemcpyAsync(s->hidden, h_host + (size_t)done * c.d, (size_t)R * c.d * 4, cudaMemcpyHostToDevice, s->st);
      hid = s->hidden;
    }
    launch(s, set_rows_kernel, dim3((R + 127) / 128), dim3(128), 0, s->crows, R, seq, pos0 + done, s->seq_len);
    mtp_forward(s, R, s->catch_tok, hid, nullptr, s->crows, false, nullptr);
    done += R;
  }
  return sync_ok(s) ? 0 : 1;
}

extern "C" int lz_mtp_prefill(const LZModel* m, LZRunState* s, const float* h_body_all, const int* next_tokens,
                              int n, int pos0) {
  if (!m || !s || !h_body_all || !next_tokens || n < 1) return 1;
  return mtp_prefill_seq(s, 0, h_body_all, nullptr, next_tokens, n, pos0);
}

extern "C" int lz_mtp_catchup(const LZModel* m, LZRunState* s, const float* h_body_all, const int* next_tokens,
                              int n, int pos0) {
  UsTimer t(&lz_debug_us_catchup);
  lz_debug_n_catchup++;
  return lz_mtp_prefill(m, s, h_body_all, next_tokens, n, pos0);
}

// ================================================================== rounds

extern "C" int lz_spec_accept(const int* draft, const int* targ, int n_draft, int bonus, int* out) {
  if (!draft || !targ || !out || n_draft < 0) return 0;     // src/generate.c:232-243
  for (int i = 0; i < n_draft; i++) {
    out[i] = targ[i];
    if (draft[i] != targ[i]) return i;
  }
  out[n_draft] = bonus;
  return n_draft;
}

static float host_random_f32(uint64_t* st) {               // src/sampler.c:185-203
  uint64_t x = *st;
  x ^= x >> 12; x ^= x << 25; x ^= x >> 27;
  *st = x;
  return (float)((unsigned)((x * 0x2545F4914F6CDD1DULL) >> 32) >> 8) / 16777216.0f;
}

static uint32_t host_fkey(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u ^ ((uint32_t)((int32_t)u >> 31) | 0x80000000u);
}

extern "C" int lz_spec_accept_temp(const float* p, const float* q, int x, int vocab, float u, uint64_t* rng,
                                   int* acc) {
  // src/generate.c:264-349
  if (!p || !q || !rng || vocab <= 0 || x < 0 || x >= vocab) {
    if (acc) *acc = 0;
    return -1;
  }
  volatile float qx = q[x], ratio;
  if (qx <= 0.0f) ratio = 0.0f;
  else {
    ratio = p[x] / qx;
    if (ratio > 1.0f) ratio = 1.0f;
  }
  if (u < ratio) {
    if (acc) *acc = 1;
    return x;
  }
  if (acc) *acc = 0;
  volatile float total = 0.0f, cdf = 0.0f;
  int last_pos = -1;
  for (int i = 0; i < vocab; i++) {
    volatile float d = p[i] - q[i];
    if (d > 0.0f) { total = total + d; last_pos = i; }
  }
  if (total <= 0.0f) {
    int mi = 0;
    uint32_t best = host_fkey(p[0]);
    for (int i = 1; i < vocab; i++) {
      uint32_t k = host_fkey(p[i]);
      if (k > best) { best = k; mi = i; }
    }
    return mi;
  }
  volatile float coin = host_random_f32(rng) * total;
  for (int i = 0; i < vocab; i++) {
    volatile float d = p[i] - q[i];
    if (d > 0.0f) {
      cdf = cdf + d;
      if (coin < cdf) return i;
    }
  }
  return last_pos;
}

static int run_round(LZRunState* s, int k) {
  const int mode = round_mode(s);
  if (mode < 0) return 1;
  if (s->graphs) {
    const int key = k + 100 * mode;
    auto it = s->graph.find(key);
    if (it == s->graph.end()) {
      cudaGraph_t g;
      CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
      round_any(s, k);
      CK(cudaStreamEndCapture(s->st, &g));
      cudaGraphExec_t ge;
      CK(cudaGraphInstantiate(&ge, g, 0));
      cudaGraphDestroy(g);
      it = s->graph.emplace(key, ge).first;
    }
    CK(cudaGraphLaunch(it->second, s->st));
  } else {
    round_any(s, k);
  }
  return 0;
}

extern "C" int lz_seq_set_sampler(LZRunState* s, int seq, float temperature, float topp, uint64_t seed) {
  if (!s || seq < 0 || seq >= s->B) return LZ98_ERR_NULL_ARG;
  if (!sr_down(s)) return LZ98_ERR_CUDA;
  SeqRound& r = s->h_sr[seq];
  r.temp = temperature > 0.0f ? temperature : 0.0f;    // src/generate.c:2790
  r.topp = topp;
  r.rng = seed ? seed : 1ull;                         // src/sampler.c:55-60
  s->seq_temp[seq] = r.temp > kTempFloor;
  return sr_up(s) && sync_ok(s) ? 0 : LZ98_ERR_CUDA;
}

extern "C" int lz_seq_get_sampler(const LZRunState* cs, int seq, float* temperature, float* topp, uint64_t* rng) {
  LZRunState* s = const_cast<LZRunState*>(cs);
  if (!s || seq < 0 || seq >= s->B) return LZ98_ERR_NULL_ARG;
  if (!sr_down(s)) return LZ98_ERR_CUDA;
  const SeqRound& r = s->h_sr[seq];
  if (temperature) *temperature = r.temp;
  if (topp) *topp = r.topp;
  if (rng) *rng = r.rng;
  return 0;
}

// Sampler options the device rounds do not carry, refused rather than
// ignored: penalties that act (the reference applies them to every verify
// row through an assumed window, src/generate.c:517-529, 639-690) and, for
// the temperature round, top-k and min-p (src/sampler.c:682-714).  The
// think temperature is not read by the rounds.
static const char* sampler_refusal(const LZSampler* sp, int vocab, bool temp) {
  const LZSampleParams& p = sp->p;
  const bool has_rep = p.repetition_penalty != 1.0f;
  const bool has_add = p.presence_penalty != 0.0f || p.frequency_penalty != 0.0f;
  if (p.repeat_last_n != 0 && (has_rep || has_add)) return "sampler penalties are not supported on the device path";
  if (!temp) return nullptr;
  if (p.topk > 0 && p.topk < vocab) return "top-k is not supported on the device path";
  if (p.minp > 0.0f) return "min-p is not supported on the device path";
  if (!(p.temperature > kTempFloor)) return "temperature round with a temperature at the greedy floor";
  return nullptr;
}

// One round of sequence 0 behind lz_spec_round (temp false) and
// lz_spec_round_temp (temp true): argument checks and refusals in the
// reference's order, the device round (captured graph) or the p_min /
// n_min round, then the reference's outputs.
static int spec_round_seq0(const LZModel* m, LZRunState* s, int anchor, int anchor_pos, int k, float p_min,
                           int n_min, const LZSampler* samp, bool temp, int dbg_break, int dbg_skip, int* out,
                           int* out_n_accept, int* out_new_pos, int* out_k_eff, uint64_t* rng_out, char* errbuf,
                           int errlen) {
  if (!m || !s || (temp && !samp) || !out || !out_n_accept || !out_new_pos || !out_k_eff) {
    set_err(errbuf, errlen, "null argument");
    return -LZ98_ERR_NULL_ARG;
  }
  if (k < 1 || k > 6 || k > s->depth - 1) {
    set_err(errbuf, errlen, "draft depth out of range");
    return -LZ98_ERR_SPEC_K_RANGE;
  }
  if (s->B != 1) {
    set_err(errbuf, errlen, "a batched state runs its rounds through lz_spec_round_batch");
    return -LZ98_ERR_FORWARD;
  }
  if (samp)
    if (const char* why = sampler_refusal(samp, m->c.vocab, temp)) {
      set_err(errbuf, errlen, "%s", why);
      return -LZ98_ERR_FORWARD;
    }
  if (!sr_down(s)) {
    round_fail(s, errbuf, errlen, "CUDA failure before the round");
    return -LZ98_ERR_CUDA;
  }
  SeqRound& r = s->h_sr[0];
  r.anchor = anchor;
  r.anchor_pos = anchor_pos;
  r.k = k;
  r.dbg = (dbg_break ? kDbgBreakRollback : 0) | (dbg_skip ? kDbgSkipCatchup : 0);
  if (temp) {
    r.temp = samp->p.temperature;
    r.topp = samp->p.topp;
    r.rng = samp->rng_state;
  } else {
    r.temp = 0.0f;
  }
  s->seq_temp[0] = temp ? 1 : 0;
  if (!sr_up(s)) {
    round_fail(s, errbuf, errlen, "CUDA failure before the round");
    return -LZ98_ERR_CUDA;
  }
  int k_eff = k;
  if (p_min > 0.0f || n_min > 0) {
    const int rc = round_pmin(s, k, temp, p_min, n_min, &k_eff);
    if (rc < 0 || !sr_down(s)) {
      round_fail(s, errbuf, errlen, "CUDA failure in the round");
      return -LZ98_ERR_CUDA;
    }
    *out_k_eff = k_eff;
    if (temp) *rng_out = s->h_sr[0].rng;   // the draft samples advanced the generator either way
    if (rc == 0) {   // draft discarded (src/generate.c:765-791)
      out[0] = anchor;
      *out_n_accept = 0;
      *out_new_pos = anchor_pos;
      return 0;
    }
  } else {
    if (run_round(s, k) || !sr_down(s)) {
      round_fail(s, errbuf, errlen, "CUDA failure in the round");
      return -LZ98_ERR_CUDA;
    }
    *out_k_eff = k;
    if (temp) *rng_out = s->h_sr[0].rng;
  }
  const SeqRound& o = s->h_sr[0];
  for (int i = 0; i <= o.n_accept; i++) out[i] = o.out[i];
  *out_n_accept = o.n_accept;
  *out_new_pos = anchor_pos + 1 + o.n_accept;
  round_debug(s, o.n_accept, k_eff);
  return o.n_accept + 1;
}

extern "C" int lz_spec_round(const LZModel* m, LZRunState* s, int anchor, int anchor_pos, int k, float p_min,
                             int n_min, const LZSampler* samp, int debug_break_rollback, int debug_skip_catchup,
                             int* out, int* out_n_accept, int* out_new_pos, int* out_k_eff, char* errbuf,
                             int errlen) {
  return spec_round_seq0(m, s, anchor, anchor_pos, k, p_min, n_min, samp, false, debug_break_rollback,
                         debug_skip_catchup, out, out_n_accept, out_new_pos, out_k_eff, nullptr, errbuf, errlen);
}

extern "C" int lz_spec_round_temp(const LZModel* m, LZRunState* s, int anchor, int anchor_pos, int k,
                                  float p_min, int n_min, LZSampler* samp, int debug_break_rollback,
                                  int debug_skip_catchup, int* out, int* out_n_accept, int* out_new_pos,
                                  int* out_k_eff, char* errbuf, int errlen) {
  uint64_t rng = samp ? samp->rng_state : 0;
  const int rc = spec_round_seq0(m, s, anchor, anchor_pos, k, p_min, n_min, samp, true, debug_break_rollback,
                                 debug_skip_catchup, out, out_n_accept, out_new_pos, out_k_eff, &rng, errbuf,
                                 errlen);
  if (rc >= 0) samp->rng_state = rng;
  return rc;
}

// Prefill of sequence `seq` with the prompt tokens at body positions
// start_pos.. (0 for a fresh sequence, the end of a restored prefix for a
// resumed one, src/generate.c:2841-2900): capture prefill, MTP prefill from
// the sequence's MTP position, capture forward of the last token and the
// first anchor.
static int seq_prefill_impl(const LZModel* m, LZRunState* s, int seq, int start_pos, const int* prompt,
                            int n_prompt, int* out_anchor, char* errbuf, int errlen) {
  if (!m || !s || !prompt || n_prompt < 1 || seq < 0 || seq >= s->B || start_pos < 0 ||
      start_pos + n_prompt >= s->seq_len) {
    set_err(errbuf, errlen, "bad prefill arguments");
    return LZ98_ERR_NULL_ARG;
  }
  const Cfg& c = m->c;
  if (!sr_down(s)) {
    round_fail(s, errbuf, errlen, "CUDA failure before prefill");
    return LZ98_ERR_CUDA;
  }
  const int slot = s->h_sr[seq].ssm_slot;
  int mtp_pos = s->h_sr[seq].mtp_pos;
  const int n = n_prompt - 1;
  if (n > 0) {
    if ((size_t)n > s->hb_rows) {
      if (s->hb) cudaFree(s->hb);
      s->hb = nullptr;
      if (cudaMalloc(&s->hb, (size_t)n * c.d * 4) != cudaSuccess) {
        set_err(errbuf, errlen, "device allocation failed");
        return LZ98_ERR_ALLOC;
      }
      s->hb_rows = n;
    }
    for (int done = 0; done < n;) {
      const int R = std::min(s->Rmax, n - done);
      cudaMemcpyAsync(s->tok, prompt + done, R * sizeof(int), cudaMemcpyHostToDevice, s->st);
      upload_seqs(s, {KdaSeq{0, R, slot, seq}});
      body_forward(s, R, 1, 0, false);
      cudaMemcpyAsync(s->hb + (size_t)done * c.d, s->hidden, (size_t)R * c.d * 4, cudaMemcpyDeviceToDevice,
                      s->st);
      done += R;
    }
    if (mtp_prefill_seq(s, seq, nullptr, s->hb, prompt + 1, n, mtp_pos)) {
      set_err(errbuf, errlen, "CUDA failure in prefill");
      return LZ98_ERR_CUDA;
    }
    mtp_pos += n;
  }
  const int last = prompt[n_prompt - 1];
  cudaMemcpyAsync(s->tok, &last, sizeof(int), cudaMemcpyHostToDevice, s->st);
  upload_seqs(s, {KdaSeq{0, 1, slot, seq}});
  body_forward(s, 1, 1, 0, true);
  cudaMemcpyAsync(s->chain + (size_t)seq * c.d, s->hidden, c.d * 4, cudaMemcpyDeviceToDevice, s->st);
  int anchor = 0;
  if (sample_row(s, seq, &anchor)) {
    set_err(errbuf, errlen, "CUDA failure in prefill");
    return LZ98_ERR_CUDA;
  }
  if (!sr_down(s)) {                 // the sampler state advanced on the device
    round_fail(s, errbuf, errlen, "CUDA failure in prefill");
    return LZ98_ERR_CUDA;
  }
  SeqRound& r = s->h_sr[seq];
  r.anchor = anchor;
  r.anchor_pos = start_pos + n_prompt - 1;
  r.mtp_pos = mtp_pos;
  r.ssm_slot = slot;
  r.dbg = 0;
  if (!sr_up(s) || !sync_ok(s)) {
    round_fail(s, errbuf, errlen, "CUDA failure in prefill");
    return LZ98_ERR_CUDA;
  }
  if (out_anchor) *out_anchor = anchor;
  return 0;
}

extern "C" int lz_seq_prefill(const LZModel* m, LZRunState* s, int seq, const int* prompt, int n_prompt,
                              int* out_anchor, char* errbuf, int errlen) {
  return seq_prefill_impl(m, s, seq, 0, prompt, n_prompt, out_anchor, errbuf, errlen);
}

extern "C" int lz_spec_round_batch(const LZModel* m, LZRunState* s, int k, int* out_tokens, int* out_counts,
                                   char* errbuf, int errlen) {
  if (!m || !s) return LZ98_ERR_NULL_ARG;
  if (k < 1 || k > s->kmax) {
    set_err(errbuf, errlen, "draft depth out of range");
    return LZ98_ERR_SPEC_K_RANGE;
  }
  if (run_round(s, k)) {
    round_fail(s, errbuf, errlen, "CUDA failure in the round");
    return LZ98_ERR_CUDA;
  }
  if (out_tokens || out_counts) {
    if (!sr_down(s)) {
      round_fail(s, errbuf, errlen, "CUDA failure in the round");
      return LZ98_ERR_CUDA;
    }
    for (int b = 0; b < s->B; b++) {
      const SeqRound& o = s->h_sr[b];
      if (out_counts) out_counts[b] = o.n_emit;
      if (out_tokens)
        for (int i = 0; i <= k; i++) out_tokens[b * (k + 1) + i] = i <= o.n_accept ? o.out[i] : -1;
    }
  } else if (cudaPeekAtLastError() != cudaSuccess || (s->h_err && *(volatile int*)s->h_err)) {
    // without a read-back the round is not waited for: launch errors and
    // a wait that gave up in an earlier round are reported here
    round_fail(s, errbuf, errlen, "CUDA failure in the round");
    return LZ98_ERR_CUDA;
  }
  return 0;
}

// The generation loop of src/generate.c:2781-3091 on token ids (sequence
// 0): greedy at the temperature floor, else coupled temperature rounds with
// top-p `topp` and the generator seeded by `seed`.  Every token is picked on
// the device.
// The generation loop of sequence 0 from body position start_pos (0 with
// a reset state: lz_generate; the end of a restored prefix: the resume
// path, src/generate.c:2781-2840).
static int generate_impl(const LZModel* m, LZRunState* s, int start_pos, bool reset, const int* prompt,
                         int n_prompt, int max_new, int spec_k, float temp, float topp, uint64_t seed, float p_min,
                         int n_min, int* out_tok, int out_cap, int* out_n, int* rounds, int round_cap,
                         int* n_rounds, char* errbuf, int errlen) {
  if (!m || !s || !prompt || n_prompt < 1 || !out_n || !n_rounds || start_pos < 0) return LZ98_ERR_NULL_ARG;
  if (start_pos + n_prompt >= s->seq_len) {
    set_err(errbuf, errlen, "prompt does not fit the state");
    return LZ98_ERR_NULL_ARG;
  }
  const Cfg& c = m->c;
  if (reset) lz_state_reset(s, m);          // src/generate.c:2813
  // the reference loop's sampler (oracle-free restatement of its settings,
  // src/generate.c:2790): temperature, top-p, identity penalties, no top-k
  // or min-p, the generator seeded with `seed` (0 taken as 1)
  LZSampler samp;
  memset(&samp, 0, sizeof samp);
  samp.vocab_size = c.vocab;
  samp.p.temperature = temp > 0.0f ? temp : 0.0f;
  samp.p.topp = topp;
  samp.p.repetition_penalty = 1.0f;
  samp.rng_state = seed ? seed : 1ull;
  const bool use_temp = samp.p.temperature > kTempFloor;
  if (int rc = lz_seq_set_sampler(s, 0, samp.p.temperature, topp, samp.rng_state)) return rc;
  int max_pos = start_pos + n_prompt + max_new;
  if (max_pos > s->seq_len) max_pos = s->seq_len;
  if (max_pos < start_pos + n_prompt + 1) max_pos = start_pos + n_prompt + 1;
  int n_out = 0, nr = 0;
  auto emit = [&](int t) { if (n_out < out_cap) out_tok[n_out] = t; n_out++; };
  int pos = start_pos + n_prompt - 1, token = prompt[n_prompt - 1];
  // one forward of `token` at `pos` in place (optionally captured into the
  // draft chain), then one token sampled by the sequence's sampler
  auto step = [&](bool capture, int* next) {
    if (!sr_down(s)) return 1;
    const int slot = s->h_sr[0].ssm_slot;
    if (cudaMemcpyAsync(s->tok, &token, sizeof(int), cudaMemcpyHostToDevice, s->st) != cudaSuccess) return 1;
    upload_seqs(s, {KdaSeq{0, 1, slot, 0}});
    body_forward(s, 1, 1, 0, true);
    if (capture) cudaMemcpyAsync(s->chain, s->hidden, c.d * 4, cudaMemcpyDeviceToDevice, s->st);
    return sample_row(s, 0, next);
  };
  // `pending` holds the anchor of a first round whose forward and sample
  // already ran (lz_seq_prefill forwards the last prompt token and picks
  // the anchor, as the first loop iteration of the reference does).
  bool have_seed = false, pending = false;
  if (spec_k > 0) {
    int rc = seq_prefill_impl(m, s, 0, start_pos, prompt, n_prompt, &token, errbuf, errlen);
    if (rc) return rc;
    emit(token);
    pending = true;
  } else if (n_prompt > 1) {
    std::vector<float> hb((size_t)(n_prompt - 1) * c.d);
    if (!lz_forward_batch_capture(m, s, prompt, n_prompt - 1, start_pos, hb.data())) return LZ98_ERR_FORWARD;
  }
  // the spec loop of lz_generate_call (src/generate.c:2841-3035, rounds by
  // src/generate.c:1900-2100)
  while (pos < max_pos - 1) {
    int round_k = 0;
    if (spec_k > 0) {
      round_k = spec_k;
      if (round_k > max_pos - 3 - pos) round_k = max_pos - 3 - pos;
    }
    if (round_k > 0) {
      int anchor, anchor_pos;
      if (have_seed || pending) {
        anchor = token;
        anchor_pos = pending ? pos : pos - 1;
      } else {
        // no seed (after a discarded draft): capture forward, fresh anchor
        if (step(true, &anchor)) return LZ98_ERR_CUDA;
        anchor_pos = pos;
        emit(anchor);
      }
      pending = false;
      int out[8], n_acc = 0, new_pos = 0, k_eff = 0;
      int ne;
      if (use_temp) {
        if (!sr_down(s)) return LZ98_ERR_CUDA;
        samp.rng_state = s->h_sr[0].rng;
        ne = lz_spec_round_temp(m, s, anchor, anchor_pos, round_k, p_min, n_min, &samp, 0, 0, out, &n_acc,
                                &new_pos, &k_eff, errbuf, errlen);
      } else {
        ne = lz_spec_round(m, s, anchor, anchor_pos, round_k, p_min, n_min, nullptr, 0, 0, out, &n_acc, &new_pos,
                           &k_eff, errbuf, errlen);
      }
      if (ne < 0) return -ne;
      if (rounds && nr < round_cap) { rounds[2 * nr] = k_eff; rounds[2 * nr + 1] = n_acc; }
      nr++;
      have_seed = ne > 0;
      if (ne > 0)
        for (int ei = 0; ei <= n_acc; ei++) emit(out[ei]);
      pos = new_pos + 1;
      token = out[n_acc];
      continue;
    }
    if (pending) {
      // the reference's plain step for this position already ran
      pending = false;
      pos++;
      continue;
    }
    // plain decode step: forward of one token, then one sampled token
    if (step(false, &token)) return LZ98_ERR_CUDA;
    emit(token);
    pos++;
  }
  *out_n = n_out;
  *n_rounds = nr;
  return 0;
}

extern "C" int lz_generate_ex(const LZModel* m, LZRunState* s, const int* prompt, int n_prompt, int max_new,
                              int spec_k, float temp, float topp, uint64_t seed, float p_min, int n_min,
                              int* out_tok, int out_cap, int* out_n, int* rounds, int round_cap, int* n_rounds,
                              char* errbuf, int errlen) {
  return generate_impl(m, s, 0, true, prompt, n_prompt, max_new, spec_k, temp, topp, seed, p_min, n_min, out_tok,
                       out_cap, out_n, rounds, round_cap, n_rounds, errbuf, errlen);
}

extern "C" int lz_generate_resume(const LZModel* m, LZRunState* s, int start_pos, const int* suffix, int n_suffix,
                                  int max_new, int spec_k, float temp, float topp, uint64_t seed, int* out_tok,
                                  int out_cap, int* out_n, int* rounds, int round_cap, int* n_rounds, char* errbuf,
                                  int errlen) {
  return generate_impl(m, s, start_pos, false, suffix, n_suffix, max_new, spec_k, temp, topp, seed, 0.0f, 0,
                       out_tok, out_cap, out_n, rounds, round_cap, n_rounds, errbuf, errlen);
}

extern "C" int lz_generate(const LZModel* m, LZRunState* s, const int* prompt, int n_prompt, int max_new,
                           int spec_k, float temp, float topp, uint64_t seed, int* out_tok, int out_cap,
                           int* out_n, int* rounds, int round_cap, int* n_rounds, char* errbuf, int errlen) {
  return lz_generate_ex(m, s, prompt, n_prompt, max_new, spec_k, temp, topp, seed, 0.0f, 0, out_tok, out_cap, out_n,
                        rounds, round_cap, n_rounds, errbuf, errlen);
}

extern "C" int lz_state_counters(const LZRunState* cs, int seq, int* rounds, int* emitted, int* accepted,
                                 int* drafted) {
  LZRunState* s = const_cast<LZRunState*>(cs);
  if (!s || seq < 0 || seq >= s->B) return LZ98_ERR_NULL_ARG;
  if (!sr_down(s)) return LZ98_ERR_CUDA;
  const SeqRound& r = s->h_sr[seq];
  if (rounds) *rounds = r.rounds;
  if (emitted) *emitted = r.emitted;
  if (accepted) *accepted = r.accepted;
  if (drafted) *drafted = r.drafted;
  return 0;
}

// One eager round of depth k with CUDA events around every int8
// GEMV launch: total GEMV device time, their algorithmic bytes, the count,
// the round's device time and its kernel count.
extern "C" int lz_profile_round(LZRunState* s, int k, double* gemv_ms, double* gemv_bytes, int* n_gemv,
                                double* round_ms, int* n_kernels) {
  if (!s || k < 1 || k > s->kmax) return LZ98_ERR_NULL_ARG;
  cudaEvent_t r0, r1;
  cudaEventCreate(&r0);
  cudaEventCreate(&r1);
  s->prof = true;
  s->prof_ev.clear();
  s->prof_bytes.clear();
  s->prof_moe_ev.clear();
  s->prof_moe_bytes.clear();
  if (round_mode(s) < 0) return LZ98_ERR_NULL_ARG;
  const long long l0 = s->launches;
  cudaEventRecord(r0, s->st);
  round_any(s, k);
  cudaEventRecord(r1, s->st);
  s->prof = false;
  if (!sync_ok(s)) return LZ98_ERR_CUDA;
  double gt = 0.0, gb = 0.0;
  for (size_t i = 0; i < s->prof_bytes.size(); i++) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, s->prof_ev[2 * i], s->prof_ev[2 * i + 1]);
    gt += ms;
    gb += s->prof_bytes[i];
  }
  for (auto e : s->prof_ev) cudaEventDestroy(e);
  s->prof_ev.clear();
  s->prof_moe_ms = s->prof_moe_b = 0.0;
  for (size_t i = 0; i < s->prof_moe_bytes.size(); i++) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, s->prof_moe_ev[2 * i], s->prof_moe_ev[2 * i + 1]);
    s->prof_moe_ms += ms;
    s->prof_moe_b += s->prof_moe_bytes[i];
  }
  s->prof_moe_n = (int)s->prof_moe_bytes.size();
  for (auto e : s->prof_moe_ev) cudaEventDestroy(e);
  s->prof_moe_ev.clear();
  float rms = 0.0f;
  cudaEventElapsedTime(&rms, r0, r1);
  cudaEventDestroy(r0);
  cudaEventDestroy(r1);
  if (gemv_ms) *gemv_ms = gt;
  if (gemv_bytes) *gemv_bytes = gb;
  if (n_gemv) *n_gemv = (int)s->prof_bytes.size();
  if (round_ms) *round_ms = rms;
  if (n_kernels) *n_kernels = (int)(s->launches - l0);
  return 0;
}

// One eager round of depth k with events around every launch: "kernel<TAB>
// microseconds" lines into buf, in launch order.  Returns the launch count.
extern "C" int lz_profile_launches(LZRunState* s, int k, char* buf, int buflen) {
  if (!s || !buf || buflen < 1 || k < 1 || k > s->kmax || round_mode(s) < 0) return -LZ98_ERR_NULL_ARG;
  s->prof_launch.clear();
  s->prof_all = true;
  round_any(s, k);
  s->prof_all = false;
  if (!sync_ok(s)) return -LZ98_ERR_CUDA;
  int used = 0;
  buf[0] = 0;
  for (auto& t : s->prof_launch) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, std::get<1>(t), std::get<2>(t));
    const char* name = "?";
    if (cudaFuncGetName(&name, std::get<0>(t)) != cudaSuccess) name = "?";
    if (used < buflen - 1) {
      const int w = snprintf(buf + used, (size_t)(buflen - used), "%s\t%.3f\n", name, ms * 1000.0f);
      used += w < 0 ? 0 : std::min(w, buflen - 1 - used);   // a cut line stays cut
    }
    cudaEventDestroy(std::get<1>(t));
    cudaEventDestroy(std::get<2>(t));
  }
  const int n = (int)s->prof_launch.size();
  s->prof_launch.clear();
  return n;
}

// The grouped-expert launches of the last lz_profile_round: summed device
// time, algorithmic bytes and launch count.
extern "C" int lz_profile_experts(const LZRunState* s, double* ms, double* bytes, int* n) {
  if (!s) return LZ98_ERR_NULL_ARG;
  if (ms) *ms = s->prof_moe_ms;
  if (bytes) *bytes = s->prof_moe_b;
  if (n) *n = s->prof_moe_n;
  return 0;
}

// ============================================================ static scratch
//
// lz_lm_head_static: logits of final-normed hidden rows without any
// allocation, for callers that cannot call cudaMalloc (a host process that
// owns no CUDA allocator of its own, code running inside another runtime's
// memory pool or under a capture-only budget).  The quantised activation
// rows this path needs live in the file-scope arrays below, sized for at
// most kStaticRows rows of at most kStaticDim columns; every GPU that loads
// this library holds them (288 KiB) until the process exits.

namespace {

constexpr int kStaticRows = 64;
constexpr int kStaticDim = 4096;

static __device__ __align__(256) int8_t g_static_xq[kStaticRows * kStaticDim];
static __device__ __align__(256) float g_static_xs[kStaticRows * kStaticDim / 32];

constexpr int kMaxDevices = 64;

// Device addresses of the two arrays, resolved once per device (the
// arrays' host-side names are not device addresses).
struct StaticScratch {
  std::once_flag once;
  cudaError_t rc = cudaSuccess;
  int8_t* xq = nullptr;
  float* xs = nullptr;
};
StaticScratch g_static[kMaxDevices];

// Per-32 quantisation of n rows (src/ops_quant.c:2152-2282).
__global__ void quant_rows_kernel(const float* __restrict__ x, int d, int8_t* xq, float* xs) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int g = warp; g < d / 32; g += nw) {
    const int i = g * 32 + lane;
    xq[(size_t)r * d + i] = warp_quant32(x[(size_t)r * d + i], &xs[(size_t)r * (d / 32) + g]);
  }
}

}  // namespace

extern "C" int lz_lm_head_static(const LZModel* m, const float* hidden, int n, float* logits, void* stream,
                                 char* errbuf, int errlen) {
  if (!m || !hidden || !logits) {
    set_err(errbuf, errlen, "lz_lm_head_static: null argument");
    return LZ98_ERR_NULL_ARG;
  }
  const Cfg& c = m->c;
  if (n < 1 || n > kStaticRows || c.d > kStaticDim) {
    char msg[160];
    snprintf(msg, sizeof msg, "lz_lm_head_static: %d rows of %d columns exceed the static scratch (%d x %d)",
             n, c.d, kStaticRows, kStaticDim);
    set_err(errbuf, errlen, "%s", msg);
    return LZ98_ERR_SIZE;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_err(errbuf, errlen, "lz_lm_head_static: no current CUDA device");
    return LZ98_ERR_CUDA;
  }
  if (dev != m->dev) {
    set_err(errbuf, errlen, "lz_lm_head_static: the current CUDA device is not the model's");
    return LZ98_ERR_DEVICE;
  }
  // One-time set-up per device, with that device current (the first call
  // on the device does it; std::call_once makes concurrent first calls
  // from several host threads wait for one resolution).
  StaticScratch& g = g_static[dev];
  std::call_once(g.once, [&g] {
    void* pq = nullptr;
    void* ps = nullptr;
    g.rc = cudaGetSymbolAddress(&pq, g_static_xq);
    if (g.rc == cudaSuccess) g.rc = cudaGetSymbolAddress(&ps, g_static_xs);
    if (g.rc == cudaSuccess && (!pq || !ps)) g.rc = cudaErrorInvalidSymbol;
    g.xq = static_cast<int8_t*>(pq);
    g.xs = static_cast<float*>(ps);
  });
  if (g.rc != cudaSuccess) {
    set_err(errbuf, errlen, "lz_lm_head_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(g.rc));
    return LZ98_ERR_CUDA;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // each launch's own status (cudaLaunchKernel), not a sticky earlier error
  const int8_t* xq = g.xq;
  const float* xs = g.xs;
  {
    int8_t* q = g.xq;
    float* sc = g.xs;
    int d = c.d;
    void* args[] = {(void*)&hidden, &d, &q, &sc};
    const cudaError_t e = cudaLaunchKernel((const void*)quant_rows_kernel, dim3(n), dim3(256), args, 0, st);
    if (e != cudaSuccess) {
      set_err(errbuf, errlen, "lz_lm_head_static: quantisation launch failed: %s", cudaGetErrorString(e));
      return LZ98_ERR_CUDA;
    }
  }
  const QW& w = m->embed;
  GemvArgs a{w.q, w.s, w.out, w.in, w.gs, xq, xs, n, logits, c.vocab, 0, nullptr, nullptr, 0, 32, nullptr, nullptr};
  const dim3 grid((w.out + kGemvWarps - 1) / kGemvWarps), blk(kGemvWarps * 32);
  const int nsb = w.in / 32;
  const int jm = nsb <= 32 ? 1 : nsb <= 64 ? 2 : 4;
  const void* kern = jm == 1 ? (const void*)gemv_q8_kernel<1, kGemvWarps, kGemvRB, false, true>
                     : jm == 2 ? (const void*)gemv_q8_kernel<2, kGemvWarps, kGemvRB, false, true>
                               : (const void*)gemv_q8_kernel<4, kGemvWarps, kGemvRB, false, true>;
  void* gargs[] = {&a};
  const cudaError_t e =
      cudaLaunchKernel(kern, grid, blk, gargs, gemv_smem_bytes(jm, kGemvWarps, kGemvRB, true, false, n, w.in), st);
  if (e != cudaSuccess) {
    set_err(errbuf, errlen, "lz_lm_head_static: lm_head launch failed: %s", cudaGetErrorString(e));
    return LZ98_ERR_CUDA;
  }
  return 0;
}

// ================================================================ test hooks

extern "C" int lz_debug_seq_sum(const float* vals, int n, int mode, float target, float* out_value, int* out_hit) {
  if (!vals || n < 0 || mode < 0 || mode > 2 || !out_value || !out_hit) return LZ98_ERR_NULL_ARG;
  float* dv = nullptr;
  float* dout = nullptr;
  if (cudaMalloc(&dv, (size_t)std::max(n, 1) * 4) != cudaSuccess) return LZ98_ERR_ALLOC;
  if (cudaMalloc(&dout, 8) != cudaSuccess) {
    cudaFree(dv);
    return LZ98_ERR_ALLOC;
  }
  int rc = 0;
  float h[2] = {0.0f, 0.0f};
  if (cudaMemcpy(dv, vals, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = LZ98_ERR_CUDA;
  if (!rc) {
    chain_probe_kernel<<<1, kSampThreads, kSampSmem>>>(dv, n, mode, target, dout);
    if (cudaMemcpy(h, dout, 8, cudaMemcpyDeviceToHost) != cudaSuccess) rc = LZ98_ERR_CUDA;
  }
  cudaFree(dv);
  cudaFree(dout);
  if (rc) return rc;
  *out_value = h[0];
  memcpy(out_hit, &h[1], 4);
  return 0;
}

extern "C" int lz_debug_sumsq_split(const float* rows, int nrows, int n, float* out) {
  if (!rows || !out) return LZ98_ERR_NULL_ARG;
  if (nrows < 1 || nrows > 4 || n < 512 || n > 4096 || n % 512) return LZ98_ERR_SIZE;
  const int smem = nrows * (2 * n + 16) * (int)sizeof(float);
  if (cudaFuncSetAttribute(sumsq_split_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return LZ98_ERR_CUDA;
  float* dv = nullptr;
  float* dout = nullptr;
  if (cudaMalloc(&dv, (size_t)nrows * n * 4) != cudaSuccess) return LZ98_ERR_ALLOC;
  if (cudaMalloc(&dout, 16) != cudaSuccess) {
    cudaFree(dv);
    return LZ98_ERR_ALLOC;
  }
  int rc = 0;
  if (cudaMemcpy(dv, rows, (size_t)nrows * n * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = LZ98_ERR_CUDA;
  if (!rc) {
    sumsq_split_probe_kernel<<<1, nrows * kSplitGroup, smem>>>(dv, nrows, n, dout);
    if (cudaMemcpy(out, dout, (size_t)nrows * 4, cudaMemcpyDeviceToHost) != cudaSuccess) rc = LZ98_ERR_CUDA;
  }
  cudaFree(dv);
  cudaFree(dout);
  return rc;
}

extern "C" int lz_debug_wait_timeout(int* out_err, double* out_ms) {
  if (!out_err) return LZ98_ERR_NULL_ARG;
  int* h = nullptr;
  int* d = nullptr;
  if (cudaHostAlloc((void**)&h, sizeof(int), cudaHostAllocMapped) != cudaSuccess) return LZ98_ERR_ALLOC;
  *h = 0;
  int rc = cudaHostGetDevicePointer((void**)&d, h, 0) == cudaSuccess ? 0 : LZ98_ERR_CUDA;
  const auto t0 = std::chrono::steady_clock::now();
  if (!rc) {
    wait_timeout_probe_kernel<<<1, 32>>>(d);
    if (cudaDeviceSynchronize() != cudaSuccess) rc = LZ98_ERR_CUDA;
  }
  if (out_ms)
    *out_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  *out_err = *(volatile int*)h;
  cudaFreeHost(h);
  return rc;
}

extern "C" int lz_debug_inject_wait_timeout(int on, double limit_ms) {
  const int skip = on ? 1 : 0;
  const unsigned long long lim =
      on ? (unsigned long long)(std::max(limit_ms, 0.001) * 1e6) : 1000000000ull;   // default: about a second
  if (cudaMemcpyToSymbol(g_dbg_skip_stage, &skip, sizeof skip) != cudaSuccess ||
      cudaMemcpyToSymbol(g_wait_limit_ns, &lim, sizeof lim) != cudaSuccess)
    return LZ98_ERR_CUDA;
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : LZ98_ERR_CUDA;
}

extern "C" int lz_debug_argmax_p1(const float* vals, int n, int* out_idx, float* out_p1) {
  if (!vals || n < 1 || !out_idx || !out_p1) return LZ98_ERR_NULL_ARG;
  float *dv = nullptr, *dout = nullptr;
  int* drec = nullptr;
  if (cudaMalloc(&dv, (size_t)n * 4) != cudaSuccess) return LZ98_ERR_ALLOC;
  if (cudaMalloc(&drec, (size_t)n * 4) != cudaSuccess || cudaMalloc(&dout, 8) != cudaSuccess) {
    cudaFree(dv);
    cudaFree(drec);
    return LZ98_ERR_ALLOC;
  }
  int rc = 0;
  float h[2] = {0.0f, 0.0f};
  if (cudaMemcpy(dv, vals, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = LZ98_ERR_CUDA;
  if (!rc) {
    argmax_p1_probe_kernel<<<1, kSampThreads, kSampSmem>>>(dv, n, drec, dout);
    if (cudaMemcpy(h, dout, 8, cudaMemcpyDeviceToHost) != cudaSuccess) rc = LZ98_ERR_CUDA;
  }
  cudaFree(dv);
  cudaFree(drec);
  cudaFree(dout);
  if (rc) return rc;
  *out_p1 = h[0];
  memcpy(out_idx, &h[1], 4);
  return 0;
}

// =============================================================== checkpoints

struct LZStateCkpt {
  const LZModel* m = nullptr;
  int8_t *hi = nullptr, *lo = nullptr;
  float *sc = nullptr, *conv = nullptr;
  size_t n_q = 0, n_conv = 0;          // element counts of one ring slot
  int pos = -1;                        // -1: never saved into
  unsigned epoch = 0;
};

extern "C" int lz_ckpt_alloc(LZStateCkpt** out, const LZModel* m, char* errbuf, int errlen) {
  if (!out || !m) {
    set_err(errbuf, errlen, "null argument");
    return LZ98_ERR_NULL_ARG;
  }
  const Cfg& c = m->c;
  LZStateCkpt* ck = new LZStateCkpt();
  ck->m = m;
  ck->n_q = (size_t)c.nl * c.nv * c.kd * c.vd;
  ck->n_conv = (size_t)c.nl * c.conv_dim * 3;
  if (cudaMalloc(&ck->hi, ck->n_q) != cudaSuccess || cudaMalloc(&ck->lo, ck->n_q) != cudaSuccess ||
      cudaMalloc(&ck->sc, ck->n_q / 32 * 4) != cudaSuccess || cudaMalloc(&ck->conv, ck->n_conv * 4) != cudaSuccess) {
    lz_ckpt_free(ck);
    set_err(errbuf, errlen, "device allocation failed");
    return LZ98_ERR_ALLOC;
  }
  *out = ck;
  return 0;
}

extern "C" void lz_ckpt_free(LZStateCkpt* ck) {
  if (!ck) return;
  cudaFree(ck->hi);
  cudaFree(ck->lo);
  cudaFree(ck->sc);
  cudaFree(ck->conv);
  delete ck;
}

extern "C" int lz_ckpt_save_seq(LZStateCkpt* ck, const LZRunState* cs, int seq, int pos, char* errbuf,
                                int errlen) {
  LZRunState* s = const_cast<LZRunState*>(cs);
  if (!ck || !s || seq < 0 || seq >= s->B || pos < 0) {
    set_err(errbuf, errlen, "null argument");
    return LZ98_ERR_NULL_ARG;
  }
  if (ck->m != s->m || ck->n_q != s->q_slot || ck->n_conv != s->conv_slot) {
    set_err(errbuf, errlen, "checkpoint does not match this model's shapes");
    return LZ98_ERR_CKPT_SHAPE;
  }
  if (!sr_down(s)) {
    set_err(errbuf, errlen, "CUDA failure while saving");
    return LZ98_ERR_CUDA;
  }
  const int slot = s->h_sr[seq].ssm_slot;   // the live slot of the ring
  const size_t oq = (size_t)seq * s->q_seq + (size_t)slot * s->q_slot;
  const size_t oc = (size_t)seq * s->conv_seq + (size_t)slot * s->conv_slot;
  if (cudaMemcpyAsync(ck->hi, s->hi + oq, ck->n_q, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess ||
      cudaMemcpyAsync(ck->lo, s->lo + oq, ck->n_q, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess ||
      cudaMemcpyAsync(ck->sc, s->sc + oq / 32, ck->n_q / 32 * 4, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess ||
      cudaMemcpyAsync(ck->conv, s->conv + oc, ck->n_conv * 4, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess ||
      !sync_ok(s)) {
    set_err(errbuf, errlen, "CUDA failure while saving");
    return LZ98_ERR_CUDA;
  }
  ck->pos = pos;
  ck->epoch = s->epoch;
  return 0;
}

extern "C" int lz_ckpt_restore_seq(const LZStateCkpt* ck, LZRunState* s, int seq, int* out_pos, char* errbuf,
                                   int errlen) {
  if (!ck || !s || seq < 0 || seq >= s->B) {
    set_err(errbuf, errlen, "null argument");
    return LZ98_ERR_NULL_ARG;
  }
  if (ck->pos < 0) {
    set_err(errbuf, errlen, "checkpoint has never been saved into");
    return LZ98_ERR_CKPT_EMPTY;
  }
  if (ck->epoch != s->epoch) {
    set_err(errbuf, errlen, "run state was reset or reallocated since the save");
    return LZ98_ERR_CKPT_STALE;
  }
  if (ck->m != s->m || ck->n_q != s->q_slot || ck->n_conv != s->conv_slot || ck->pos >= s->seq_len) {
    set_err(errbuf, errlen, "checkpoint does not match this model's shapes");
    return LZ98_ERR_CKPT_SHAPE;
  }
  const size_t oq = (size_t)seq * s->q_seq, oc = (size_t)seq * s->conv_seq;   // ring slot 0
  if (cudaMemcpyAsync(s->hi + oq, ck->hi, ck->n_q, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess ||
      cudaMemcpyAsync(s->lo + oq, ck->lo, ck->n_q, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess ||
      cudaMemcpyAsync(s->sc + oq / 32, ck->sc, ck->n_q / 32 * 4, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess ||
      cudaMemcpyAsync(s->conv + oc, ck->conv, ck->n_conv * 4, cudaMemcpyDeviceToDevice, s->st) != cudaSuccess) {
    set_err(errbuf, errlen, "CUDA failure while restoring");
    return LZ98_ERR_CUDA;
  }
  const bool ok = sr_down(s);
  s->h_sr[seq].ssm_slot = 0;
  if (!ok || !sr_up(s) || !sync_ok(s)) {
    set_err(errbuf, errlen, "CUDA failure while restoring");
    return LZ98_ERR_CUDA;
  }
  if (out_pos) *out_pos = ck->pos;
  return 0;
}

extern "C" int lz_ckpt_save(LZStateCkpt* ck, const LZRunState* s, const LZModel* m, int pos, char* errbuf,
                            int errlen) {
  if (ck && s && m && m != s->m) {
    set_err(errbuf, errlen, "checkpoint does not match this model's shapes");
    return LZ98_ERR_CKPT_SHAPE;
  }
  return lz_ckpt_save_seq(ck, s, 0, pos, errbuf, errlen);
}

extern "C" int lz_ckpt_restore(const LZStateCkpt* ck, LZRunState* s, const LZModel* m, int* out_pos, char* errbuf,
                               int errlen) {
  if (ck && s && m && m != s->m) {
    set_err(errbuf, errlen, "checkpoint does not match this model's shapes");
    return LZ98_ERR_CKPT_SHAPE;
  }
  return lz_ckpt_restore_seq(ck, s, 0, out_pos, errbuf, errlen);
}

// ====================================================== expert parallelism

extern "C" int lz_ep_unique_id(uint8_t* out, char* errbuf, int errlen) {
  if (!out) {
    set_err(errbuf, errlen, "null argument");
    return LZ98_ERR_NULL_ARG;
  }
  const NcclApi* n = nccl_api();
  if (!n) {
    set_err(errbuf, errlen, "NCCL (libnccl.so.2) not loadable");
    return LZ98_ERR_CUDA;
  }
  ncclUniqueId id;
  const ncclResult_t r = n->get_unique_id(&id);
  if (r != ncclSuccess) {
    set_err(errbuf, errlen, "ncclGetUniqueId: %s", n->error_string(r));
    return LZ98_ERR_CUDA;
  }
  memcpy(out, &id, sizeof id);
  return 0;
}

extern "C" int lz_ep_init(LZRunState* s, const uint8_t* id, int rank, int world, char* errbuf, int errlen) {
  if (!s || !id || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world) {
    set_err(errbuf, errlen, "bad expert-parallel arguments (1 <= world <= 8, 0 <= rank < world)");
    return LZ98_ERR_NULL_ARG;
  }
  const Cfg& c = s->m->c;
  if (s->ep.comm) {
    set_err(errbuf, errlen, "expert parallelism is already set up on this state");
    return LZ98_ERR_NULL_ARG;
  }
  if (c.ne % world) {
    set_err(errbuf, errlen, "the expert count does not split evenly over the ranks");
    return LZ98_ERR_SIZE;
  }
  const int cap = s->Rmax * c.topk;           // pairs of one rank's forward at most
  if ((long)world * cap > 1024L * kMoeGroupPer) {
    set_err(errbuf, errlen, "too many pairs per layer for the expert-parallel grouping (world x rows x top-k)");
    return LZ98_ERR_SIZE;
  }
  const NcclApi* n = nccl_api();
  if (!n) {
    set_err(errbuf, errlen, "NCCL (libnccl.so.2) not loadable");
    return LZ98_ERR_CUDA;
  }
  EpCtx& E = s->ep;
  E.world = world;
  E.rank = rank;
  E.epr = c.ne / world;
  E.e0 = rank * E.epr;
  E.buf.world = world;
  E.buf.rank = rank;
  E.buf.cap = cap;
  E.buf.latent = c.latent;
  E.buf.slot_bytes = ((size_t)c.latent + (size_t)c.latent / 32 * 4 + 8 + 15) & ~(size_t)15;
  E.buf.buf_bytes = 16 + (size_t)cap * E.buf.slot_bytes;
  const size_t W = world, Pr = (size_t)world * cap;
  bool ok = dmalloc(s, &E.buf.send, W * E.buf.buf_bytes) && dmalloc(s, &E.buf.recv, W * E.buf.buf_bytes) &&
            dmalloc(s, &E.pair_dest, cap) && dmalloc(s, &E.pair_slot, cap) && dmalloc(s, &E.expert, Pr) &&
            dmalloc(s, &E.src, Pr) && dmalloc(s, &E.slot, Pr) && dmalloc(s, &E.total, 1) && dmalloc(s, &E.list, Pr) &&
            dmalloc(s, &E.ntiles, 1) && dmalloc(s, &E.tiles, Pr + E.epr + 1) && dmalloc(s, &E.latq, Pr * c.latent) &&
            dmalloc(s, &E.lats, Pr * c.latent / 32) && dmalloc(s, &E.hq, Pr * c.moe_ffn) &&
            dmalloc(s, &E.hs, Pr * c.moe_ffn / 32) && dmalloc(s, &E.h2, Pr * c.latent) &&
            dmalloc(s, &E.sendback, Pr * c.latent) && dmalloc(s, &E.recvback, Pr * c.latent);
  if (!ok || cudaDeviceSynchronize() != cudaSuccess) {
    E = EpCtx{};
    set_err(errbuf, errlen, "device allocation failed");
    return LZ98_ERR_ALLOC;
  }
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = n->comm_init_rank(&comm, world, uid, rank);   // every rank calls this together
  if (r != ncclSuccess) {
    E = EpCtx{};
    set_err(errbuf, errlen, "ncclCommInitRank: %s", n->error_string(r));
    return LZ98_ERR_CUDA;
  }
  E.comm = comm;
  // the exchanges run eagerly (no graph capture)
  for (auto& kv : s->graph) cudaGraphExecDestroy(kv.second);
  s->graph.clear();
  s->graphs = false;
  return 0;
}

// ============================================================== prefix cache
//
// The reference's LZPrefixCache (src/llama_zh.h:781-888,
// src/generate.c:3209-3390) on token ids: one conversation's reusable
// prefix as a device checkpoint of the recurrent state plus the token
// sequence it covers.  The render/tokenizer half of lz_prefix_prepare stays
// with the caller, who passes the three encodings (whole render, the part
// before the split, the part after it); the checks and the state work are
// the reference's, in its order.

struct LZPrefixCache {
  const LZModel* m = nullptr;
  LZStateCkpt* ck = nullptr;
  std::vector<int> tok;   // the covered token prefix
  int n = 0;              // tokens covered; 0 = nothing cached
  int have = 0;           // a checkpoint has been saved
  long n_calls = 0, n_hits = 0, n_tokens_saved = 0, n_mismatch = 0, n_unsplittable = 0;
};

extern "C" int lz_prefix_init(LZPrefixCache** out, const LZModel* m, char* errbuf, int errlen) {
  if (!out || !m) {
    set_err(errbuf, errlen, "null argument");
    return LZ98_ERR_NULL_ARG;
  }
  *out = nullptr;
  LZPrefixCache* pc = new LZPrefixCache();
  pc->m = m;
  if (int rc = lz_ckpt_alloc(&pc->ck, m, errbuf, errlen)) {
    delete pc;
    return rc;
  }
  *out = pc;
  return 0;
}

extern "C" void lz_prefix_free(LZPrefixCache* pc) {
  if (!pc) return;
  lz_ckpt_free(pc->ck);
  delete pc;
}

extern "C" void lz_prefix_reset(LZPrefixCache* pc) {
  if (!pc) return;
  pc->n = 0;
  pc->have = 0;
}

extern "C" int lz_prefix_match(const LZPrefixCache* pc, const int* pre, int n_pre) {
  if (!pc || !pre || n_pre <= 0) return 0;
  if (!pc->have || pc->n <= 0 || pc->n > n_pre) return 0;
  if (memcmp(pre, pc->tok.data(), (size_t)pc->n * sizeof(int)) != 0) return 0;
  return pc->n;
}

extern "C" int lz_prefix_prepare_tokens(LZPrefixCache* pc, const LZModel* m, LZRunState* s, const int* cur,
                                        int n_cur, const int* pre, int n_pre, const int* tail, int n_tail,
                                        int* out_start_pos, int* out_reused, char* errbuf, int errlen) {
  if (out_start_pos) *out_start_pos = 0;
  if (out_reused) *out_reused = 0;
  if (!pc || !m || !s || !cur || n_cur < 0 || (n_pre > 0 && !pre) || (n_tail > 0 && !tail)) {
    set_err(errbuf, errlen, "null argument");
    return LZ98_ERR_NULL_ARG;
  }
  pc->n_calls++;
  // nothing to reuse: the full path (not an error)
  if (n_pre <= 0 || n_tail <= 0) return 0;
  // check 1: the split is token-exact
  if (n_cur <= 0 || n_pre + n_tail != n_cur || memcmp(cur, pre, (size_t)n_pre * sizeof(int)) != 0 ||
      memcmp(cur + n_pre, tail, (size_t)n_tail * sizeof(int)) != 0) {
    pc->n_unsplittable++;
    lz_prefix_reset(pc);
    return 0;
  }
  if (n_pre >= s->seq_len) {
    set_err(errbuf, errlen, "prefix does not fit the state");
    return LZ98_ERR_NULL_ARG;
  }
  // check 2: the cached prefix is a prefix of this render (check 3, the
  // state not reset since the save, is the checkpoint's epoch test)
  int base = 0;
  if (lz_prefix_match(pc, cur, n_pre) > 0) {
    int p = 0;
    if (lz_ckpt_restore(pc->ck, s, m, &p, nullptr, 0) == 0 && p == pc->n) {
      base = pc->n;
      pc->n_hits++;
      pc->n_tokens_saved += base;
    } else {
      pc->have = 0;   // stale: rebuild from scratch
    }
  } else if (pc->have) {
    pc->n_mismatch++;
  }
  if (base == 0) lz_state_reset(s, m);
  if (n_pre > base && !forward_one(m, s, cur + base, n_pre - base, base, false, nullptr, false)) {
    // the state is half-forwarded and the cache would describe a prefix
    // that is not there: both are torn down
    lz_state_reset(s, m);
    lz_prefix_reset(pc);
    set_err(errbuf, errlen, "forward of the prefix failed");
    return LZ98_ERR_FORWARD;
  }
  // cache this render's prefix for the next turn (a failed save only loses
  // the reuse next time)
  if (lz_ckpt_save(pc->ck, s, m, n_pre, nullptr, 0) == 0) {
    pc->tok.assign(cur, cur + n_pre);
    pc->n = n_pre;
    pc->have = 1;
  } else {
    pc->have = 0;
  }
  if (out_start_pos) *out_start_pos = n_pre;
  if (out_reused) *out_reused = base;
  return 0;
}

extern "C" void lz_prefix_stats(const LZPrefixCache* pc, long* calls, long* hits, long* tokens_saved, long* mismatch,
                                long* unsplittable) {
  if (calls) *calls = pc ? pc->n_calls : 0;
  if (hits) *hits = pc ? pc->n_hits : 0;
  if (tokens_saved) *tokens_saved = pc ? pc->n_tokens_saved : 0;
  if (mismatch) *mismatch = pc ? pc->n_mismatch : 0;
  if (unsplittable) *unsplittable = pc ? pc->n_unsplittable : 0;
}
