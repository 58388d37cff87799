// Persistent device-weight cache (C++14).
//
// A model's device form (f16 B operands padded for TMA, block-form q4_0 / q8_0 planes, folded neck and
// fused projection weights, tables computed at load) takes host work the reference redoes at every
// start (sam3_load_tensors, sam3.cpp:3091-3194: each tensor read and converted). After one normal load,
// s3b_load_model_cached writes that device form to a cache file: a header that identifies the source
// file (size, modification time, a hash of its first and last MiB), the engine's format id and the
// load options that shape it, then every field of the model in one fixed order (one visitor serves
// both directions), device buffers as their bytes. A later load whose header matches maps the file and
// copies the buffers straight to the device with no conversion; any mismatch or damage falls back to
// the normal load, which rewrites the cache.
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <vector>

#include "engine.h"

namespace s3b {

namespace {

constexpr char kMagic[8] = {'S', '3', 'B', 'W', 'C', 'A', 'C', 'H'};
constexpr uint32_t kFormat = 1;  // bump when the Model layout or a buffer's device form changes

struct CacheHeader {
  char magic[8];
  uint32_t format;
  int32_t weights_quantised;
  uint64_t src_size;
  int64_t src_mtime_ns;
  uint64_t src_hash;
  uint64_t payload_bytes;
};

uint64_t fnv1a(const uint8_t* p, size_t n, uint64_t h) {
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 1099511628211ULL;
  }
  return h;
}

// size, mtime and a hash of the first and last MiB of the source file
bool source_id(const std::string& path, CacheHeader& h) {
  struct stat st;
  if (stat(path.c_str(), &st) != 0) return false;
  h.src_size = (uint64_t)st.st_size;
  h.src_mtime_ns = (int64_t)st.st_mtim.tv_sec * 1000000000LL + st.st_mtim.tv_nsec;
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  std::vector<uint8_t> buf(1 << 20);
  uint64_t hash = 1469598103934665603ULL;
  size_t n = fread(buf.data(), 1, buf.size(), f);
  hash = fnv1a(buf.data(), n, hash);
  if (h.src_size > buf.size()) {
    fseek(f, -(long)buf.size(), SEEK_END);
    n = fread(buf.data(), 1, buf.size(), f);
    hash = fnv1a(buf.data(), n, hash);
  }
  fclose(f);
  h.src_hash = hash;
  return true;
}

// Serialising side: fields appended to a host byte stream, device buffers copied back first.
struct Writer {
  std::vector<uint8_t> out;
  bool ok = true;
  void raw(const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    out.insert(out.end(), b, b + n);
  }
  template <typename T>
  void pod(T& v) {
    raw(&v, sizeof(T));
  }
  void dev(std::shared_ptr<DevBuf>& b) {
    uint64_t n = (b && b->p) ? b->bytes : 0;
    uint8_t present = b ? 1 : 0;
    pod(present);
    pod(n);
    if (!n) return;
    const size_t at = out.size();
    out.resize(at + n);
    if (cudaMemcpy(out.data() + at, b->p, n, cudaMemcpyDeviceToHost) != cudaSuccess) ok = false;
  }
  void host(std::vector<float>& v) {
    uint64_t n = v.size();
    pod(n);
    raw(v.data(), n * sizeof(float));
  }
  template <typename T, typename F>
  void vec(std::vector<T>& v, F each) {
    uint64_t n = v.size();
    pod(n);
    for (T& x : v) each(x);
  }
};

// Deserialising side: fields read from the mapped file; device buffers are allocated while parsing and
// their bytes queued, then streamed to the device through two pinned staging halves (stream_uploads).
struct Reader {
  s3b_ctx* ctx;
  const uint8_t* p;
  size_t left;
  bool ok = true;
  struct Pending {
    void* dst;
    const uint8_t* src;
    size_t n;
  };
  std::vector<Pending> uploads;
  void raw(void* dst, size_t n) {
    if (!ok || n > left) {
      ok = false;
      return;
    }
    memcpy(dst, p, n);
    p += n;
    left -= n;
  }
  template <typename T>
  void pod(T& v) {
    raw(&v, sizeof(T));
  }
  void dev(std::shared_ptr<DevBuf>& b) {
    uint8_t present = 0;
    uint64_t n = 0;
    pod(present);
    pod(n);
    if (!ok) return;
    b.reset();
    if (!present) return;
    b = std::make_shared<DevBuf>();
    if (!n) return;
    if (n > left || b->reserve(n) != 0) {
      ok = false;
      return;
    }
    uploads.push_back({b->p, p, (size_t)n});
    ctx->model.device_bytes += n;
    p += n;
    left -= n;
  }
  void host(std::vector<float>& v) {
    uint64_t n = 0;
    pod(n);
    if (!ok || n * sizeof(float) > left) {
      ok = false;
      return;
    }
    v.resize(n);
    raw(v.data(), n * sizeof(float));
  }
  template <typename T, typename F>
  void vec(std::vector<T>& v, F each) {
    uint64_t n = 0;
    pod(n);
    if (!ok || n > (1u << 20)) {
      ok = false;
      return;
    }
    v.resize(n);
    for (T& x : v) each(x);
  }
};

// The queued buffers in file order through two pinned staging halves of 32 MiB: the host fills one half
// while the copy engine drains the other; an event per half orders the reuse.
bool stream_uploads(s3b_ctx* ctx, const std::vector<Reader::Pending>& ups) {
  constexpr size_t kHalf = 32u << 20;
  uint8_t* pin = nullptr;
  if (cudaMallocHost(&pin, 2 * kHalf) != cudaSuccess) return false;
  cudaEvent_t ev[2];
  cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming);
  cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming);
  bool ok = true, used[2] = {false, false};
  int half = 0;
  size_t fill = 0;
  struct Seg {
    void* dst;
    size_t off, n;
  };
  std::vector<Seg> segs;
  auto flush = [&]() {
    for (const Seg& g : segs)
      if (cudaMemcpyAsync(g.dst, pin + half * kHalf + g.off, g.n, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess)
        ok = false;
    cudaEventRecord(ev[half], ctx->stream);
    used[half] = true;
    segs.clear();
    half ^= 1;
    fill = 0;
    if (used[half]) cudaEventSynchronize(ev[half]);
  };
  for (const Reader::Pending& u : ups) {
    size_t done = 0;
    while (done < u.n && ok) {
      if (fill == kHalf) flush();
      const size_t take = std::min(u.n - done, kHalf - fill);
      memcpy(pin + half * kHalf + fill, u.src + done, take);
      segs.push_back({static_cast<uint8_t*>(u.dst) + done, fill, take});
      fill += take;
      done += take;
    }
  }
  if (fill) flush();
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) ok = false;
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  cudaFreeHost(pin);
  return ok;
}

// Every field of the model, in one order for both directions.
template <typename IO>
void io_linear(IO& io, Linear& L) {
  io.pod(L.N);
  io.pod(L.K);
  io.pod(L.Kpad);
  io.pod(L.file_dtype);
  io.dev(L.w);
  io.dev(L.b);
  io.dev(L.raw);
  io.pod(L.qtype);
  io.dev(L.qv);
  io.dev(L.qs);
}

template <typename IO>
void io_vec(IO& io, Vec& v) {
  io.dev(v.d);
  io.pod(v.n);
}

template <typename IO>
void io_model(IO& io, Model& M) {
  io.pod(M.hp);
  io_linear(io, M.patch);
  io.dev(M.pos_tiled);
  io_vec(io, M.ln_pre_w);
  io_vec(io, M.ln_pre_b);
  io.vec(M.vit, [&](VitBlock& B) {
    io_vec(io, B.n1w);
    io_vec(io, B.n1b);
    io_vec(io, B.n2w);
    io_vec(io, B.n2b);
    io_linear(io, B.qkv);
    io_linear(io, B.proj);
    io_linear(io, B.fc1);
    io_linear(io, B.fc2);
    io.dev(B.rope);
    io.pod(B.rope_n);
    io.pod(B.global);
  });
  for (int s = 0; s < 4; ++s)
    for (NeckScale* n : {&M.neck_trk[s], &M.neck_det[s]}) {
      io_linear(io, n->dc1);
      io_linear(io, n->dcf);
      io_linear(io, n->c1);
      io_linear(io, n->c3);
    }
  io.pod(M.has_neck_trk);
  io.pod(M.has_neck_det);
  io_linear(io, M.hpatch);
  io.host(M.pos_bkg);
  io.host(M.pos_win);
  io.dev(M.hiera_pe);
  io.pod(M.hiera_pe_size);
  io.vec(M.hiera, [&](HieraBlock& B) {
    io_vec(io, B.n1w);
    io_vec(io, B.n1b);
    io_vec(io, B.n2w);
    io_vec(io, B.n2b);
    io_linear(io, B.qkv);
    io_linear(io, B.proj);
    io_linear(io, B.fc1);
    io_linear(io, B.fc2);
    io_linear(io, B.dim_proj);
    io.pod(B.dim_in);
    io.pod(B.dim_out);
    io.pod(B.heads);
    io.pod(B.window);
    io.pod(B.stage);
    io.pod(B.q_stride);
    io.pod(B.has_dim_proj);
  });
  for (int i = 0; i < 4; ++i) io.pod(M.stage_ends[i]);
  for (int i = 0; i < 4; ++i) io_linear(io, M.fpn[i]);
  io.vec(M.mem, [&](MemAttnLayer& L) {
    for (Vec* v : {&L.n1w, &L.n1b, &L.n2w, &L.n2b, &L.n3w, &L.n3b}) io_vec(io, *v);
    for (Linear* l : {&L.sa_qkv, &L.sa_out, &L.ca_q, &L.ca_k, &L.ca_v, &L.ca_out, &L.fc1, &L.fc2}) io_linear(io, *l);
  });
  io_vec(io, M.mem_norm_w);
  io_vec(io, M.mem_norm_b);
  io.pod(M.has_mem_attn);
  io.host(M.maskmem_tpos);
  io.host(M.obj_ptr_tpos_w);
  io.host(M.obj_ptr_tpos_b);
  // mask decoder
  SamDecoder& d = M.dec;
  io.pod(d.loaded);
  io.pod(d.D);
  io.pod(d.n_mask);
  io.pod(d.has_obj);
  io.pod(d.heads);
  io.vec(d.blocks, [&](SamTwoWay& B) {
    for (Linear* l : {&B.sa_q, &B.sa_k, &B.sa_v, &B.sa_out, &B.t2i_q, &B.t2i_out, &B.kq, &B.t2i_v, &B.i2t_k, &B.i2t_v,
                      &B.i2t_out, &B.mlp1, &B.mlp2})
      io_linear(io, *l);
    for (Vec* v : {&B.n1w, &B.n1b, &B.n2w, &B.n2b, &B.n3w, &B.n3b, &B.n4w, &B.n4b}) io_vec(io, *v);
  });
  for (Linear* l : {&d.fin_q, &d.fin_k, &d.fin_v, &d.fin_out, &d.up1, &d.up2, &d.conv_s0, &d.conv_s1}) io_linear(io, *l);
  for (Vec* v : {&d.fin_nw, &d.fin_nb, &d.up1_nw, &d.up1_nb}) io_vec(io, *v);
  io.vec(d.hyper, [&](Linear& l) { io_linear(io, l); });
  for (int j = 0; j < 3; ++j) {
    io_linear(io, d.iou[j]);
    io_linear(io, d.obj[j]);
  }
  io.host(d.pe_gauss);
  for (int i = 0; i < 4; ++i) io.host(d.point_emb[i]);
  io.host(d.not_a_point);
  io.host(d.no_mask);
  io.host(d.no_mem);
  io.dev(d.tokens);
  for (Vec* v : {&d.d_no_mask, &d.d_no_mem, &d.d_not_a_point}) io_vec(io, *v);
  // memory encoder + object pointer
  MemEncoder& e = M.menc;
  io.pod(e.loaded);
  io.pod(e.D);
  io.pod(e.MD);
  for (int s = 0; s < 3; ++s) {
    io_vec(io, e.ds_w[s]);
    io_vec(io, e.ds_b[s]);
  }
  io_linear(io, e.ds3);
  for (int s = 0; s < 4; ++s) {
    io_vec(io, e.ds_nw[s]);
    io_vec(io, e.ds_nb[s]);
  }
  io_linear(io, e.ds12);
  io_linear(io, e.pix);
  for (int i = 0; i < 2; ++i) {
    for (Vec* v : {&e.fuser[i].dw, &e.fuser[i].dw_b, &e.fuser[i].nw, &e.fuser[i].nb}) io_vec(io, *v);
    io_linear(io, e.fuser[i].fc1);
    io_linear(io, e.fuser[i].fc2);
  }
  io_linear(io, e.out);
  io_vec(io, e.no_obj_spatial);
  for (int j = 0; j < 3; ++j) io_linear(io, e.ptr[j]);
  io_vec(io, e.no_obj_ptr);
  io.pod(e.sig_scale);
  io.pod(e.sig_bias);
  io.pod(M.qstage_elems);
}

int read_cache(s3b_ctx* ctx, const std::string& cache_path, const CacheHeader& want) {
  const int fd = open(cache_path.c_str(), O_RDONLY);
  if (fd < 0) return 1;
  struct stat st;
  if (fstat(fd, &st) != 0 || (size_t)st.st_size < sizeof(CacheHeader)) {
    close(fd);
    return 1;
  }
  void* map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) return 1;
  CacheHeader h;
  memcpy(&h, map, sizeof h);
  int rc = 1;
  if (memcmp(h.magic, kMagic, 8) == 0 && h.format == want.format && h.weights_quantised == want.weights_quantised &&
      h.src_size == want.src_size && h.src_mtime_ns == want.src_mtime_ns && h.src_hash == want.src_hash &&
      h.payload_bytes == (uint64_t)st.st_size - sizeof(CacheHeader)) {
    ctx->model = Model();
    Reader r{ctx, static_cast<const uint8_t*>(map) + sizeof(CacheHeader), (size_t)h.payload_bytes};
    io_model(r, ctx->model);
    rc = (r.ok && r.left == 0 && stream_uploads(ctx, r.uploads)) ? 0 : 1;
    if (rc) ctx->model = Model();  // damaged: the caller rebuilds from the model file
  }
  munmap(map, (size_t)st.st_size);
  return rc;
}

int write_cache(s3b_ctx* ctx, const std::string& cache_path, CacheHeader h) {
  Writer w;
  io_model(w, ctx->model);
  if (!w.ok) return set_error(ctx, kErrCuda, "weight cache: device read-back failed");
  h.payload_bytes = w.out.size();
  const std::string tmp = cache_path + ".tmp" + std::to_string((long)getpid());
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return set_error(ctx, kErrIO, "weight cache: cannot write %s", tmp.c_str());
  const bool ok = fwrite(&h, sizeof h, 1, f) == 1 && fwrite(w.out.data(), 1, w.out.size(), f) == w.out.size();
  if (fclose(f) != 0 || !ok || rename(tmp.c_str(), cache_path.c_str()) != 0) {
    unlink(tmp.c_str());
    return set_error(ctx, kErrIO, "weight cache: writing %s failed", cache_path.c_str());
  }
  return kOk;
}

}  // namespace

int load_model_cached(s3b_ctx* ctx, const std::string& model_path, const std::string& cache_path) {
  CacheHeader h;
  memset(&h, 0, sizeof h);
  memcpy(h.magic, kMagic, 8);
  h.format = kFormat;
  h.weights_quantised = ctx->weights_quantised;
  if (!source_id(model_path, h)) return set_error(ctx, kErrIO, "cannot open %s", model_path.c_str());
  cudaSetDevice(ctx->device);
  if (read_cache(ctx, cache_path, h) == 0) {
    int rc = 0;
    if (const size_t elems = stage_arena_elems(ctx->model)) {
      ctx->buf("wq_stage", elems * 2, &rc);
      if (!rc) ctx->buf("wq_stage1", ctx->model.qstage_elems * 2, &rc);
      if (rc) return rc;
    }
    ctx->model.loaded = true;
    return 1;
  }
  int rc = load_model(ctx, model_path);
  if (rc) return rc;
  // a cache that cannot be written leaves a loaded model; the message tells why
  if (write_cache(ctx, cache_path, h) != kOk)
    fprintf(stderr, "s3b_load_model_cached: %s (the model is loaded)\n", ctx->last_error.c_str());
  return kOk;
}

}  // namespace s3b
