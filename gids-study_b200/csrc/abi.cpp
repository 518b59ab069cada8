// extern "C" entry points of libgids_b200.so (declared in include/gids_b200.h).
// Each wraps one Store/Controllers method, converts exceptions into negative
// error codes and records the message for gids_last_error().
#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <new>
#include <string>

#include "gids_internal.hpp"

struct gids_ctrls {
  gids::Controllers c;
};
struct gids_store {
  explicit gids_store(uint32_t eb, int dev) : s(eb, dev) {}
  gids::Store s;
};
struct gids_sampler {
  gids::Sampler* p = nullptr;
  ~gids_sampler() { gids::sampler_destroy(p); }
};

gids::Store* gids_store_of(gids_store_t* s) { return &s->s; }

namespace gids {
namespace {
thread_local std::string g_last_error;
}
void set_last_error(const std::string& m) { g_last_error = m; }
void clear_last_error() { g_last_error.clear(); }
}  // namespace gids

namespace {
template <typename F>
int guarded(F&& f) {
  try {
    f();
    gids::clear_last_error();
    return GIDS_OK;
  } catch (const gids::Error& e) {
    gids::set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    gids::set_last_error("host allocation failed");
    return GIDS_E_NOMEM;
  } catch (const std::exception& e) {
    gids::set_last_error(e.what());
    return GIDS_E_INVAL;
  } catch (...) {
    gids::set_last_error("unknown error");
    return GIDS_E_INVAL;
  }
}
#define NEED(p) GIDS_CHECK((p) != nullptr, GIDS_E_INVAL, #p " is null")
}  // namespace

extern "C" {

int gids_last_error(char* buf, size_t len) {
  const std::string& m = gids::g_last_error;
  if (buf && len) {
    const size_t n = m.size() < len - 1 ? m.size() : len - 1;
    memcpy(buf, m.data(), n);
    buf[n] = 0;
  }
  return (int)m.size();
}

const char* gids_strerror(int code) {
  switch (code) {
    case GIDS_OK: return "ok";
    case GIDS_E_INVAL: return "invalid argument";
    case GIDS_E_CUDA: return "CUDA error";
    case GIDS_E_NOMEM: return "out of memory";
    case GIDS_E_STATE: return "call out of order";
    case GIDS_E_RANGE: return "node id out of range";
    case GIDS_E_IO: return "emulated SSD I/O error";
    case GIDS_E_UNSUPPORTED: return "unsupported";
    default: return "unknown error code";
  }
}

const char* gids_version(void) { return "gids_b200 0.1 (sm_100a)"; }

int gids_current_device(int* out) {
  return guarded([&] {
    NEED(out);
    GIDS_CUDA(cudaGetDevice(out));
  });
}

int gids_ctrls_create(gids_ctrls_t** out) {
  return guarded([&] {
    NEED(out);
    *out = new gids_ctrls();
  });
}

int gids_ctrls_init(gids_ctrls_t* c, uint32_t n, uint64_t qd, uint64_t nq, const int32_t* list) {
  return guarded([&] {
    NEED(c);
    c->c.init(n, qd, nq, list);
  });
}

int gids_ctrls_set_emulation(gids_ctrls_t* c, uint64_t cap, const char* pattern) {
  return guarded([&] {
    NEED(c);
    c->c.set_emulation(cap, pattern);
  });
}

int gids_ctrls_destroy(gids_ctrls_t* c) {
  return guarded([&] { delete c; });
}

int gids_ctrls_bind(gids_ctrls_t* c, uint32_t num_ssd, uint32_t page_size, uint64_t read_off_pages,
                    uint64_t range_bytes) {
  return guarded([&] {
    NEED(c);
    GIDS_CHECK(page_size >= 512 && (page_size & (page_size - 1)) == 0, GIDS_E_INVAL,
               "page_size must be a power of two >= 512");
    GIDS_CHECK(num_ssd >= 1 && num_ssd <= c->c.n_ctrls, GIDS_E_INVAL, "num_ssd must be in [1, controllers]");
    GIDS_CHECK(range_bytes > 0, GIDS_E_INVAL, "empty range");
    c->c.bind(num_ssd, page_size, read_off_pages, (range_bytes + page_size - 1) / page_size);
  });
}

int gids_ctrls_write(gids_ctrls_t* c, const void* src, uint64_t nbytes, uint64_t off) {
  return guarded([&] {
    NEED(c);
    GIDS_CHECK(c->c.bound, GIDS_E_STATE, "controllers not bound");
    GIDS_CHECK(off + nbytes <= c->c.range_pages * c->c.page_size, GIDS_E_RANGE, "write past the end of the range");
    if (nbytes) NEED(src);
    gids::backing_write(c->c, src, nbytes, off);
  });
}

int gids_ctrls_read(gids_ctrls_t* c, void* dst, uint64_t nbytes, uint64_t off) {
  return guarded([&] {
    NEED(c);
    GIDS_CHECK(c->c.bound, GIDS_E_STATE, "controllers not bound");
    GIDS_CHECK(off + nbytes <= c->c.range_pages * c->c.page_size, GIDS_E_RANGE, "read past the end of the range");
    if (nbytes) NEED(dst);
    gids::backing_read(c->c, dst, nbytes, off);
  });
}

int gids_ctrls_fill_synthetic(gids_ctrls_t* c, int kind, uint64_t seed, int threads) {
  return guarded([&] {
    NEED(c);
    GIDS_CHECK(c->c.bound, GIDS_E_STATE, "controllers not bound");
    gids::backing_fill_synthetic(c->c, kind, seed, threads);
  });
}

int gids_ctrls_geometry(gids_ctrls_t* c, uint64_t* out, int count) {
  return guarded([&] {
    NEED(c);
    NEED(out);
    GIDS_CHECK(c->c.bound, GIDS_E_STATE, "controllers not bound");
    const uint64_t g[4] = {c->c.range_pages, c->c.wrap_pages, c->c.ssd.empty() ? 0 : c->c.ssd[0].bytes,
                           c->c.n_bound};
    for (int i = 0; i < count && i < 4; i++) out[i] = g[i];
  });
}

int gids_store_create(gids_store_t** out, uint32_t elem_bytes, int device) {
  return guarded([&] {
    NEED(out);
    *out = new gids_store(elem_bytes, device);
  });
}

int gids_store_init_controllers(gids_store_t* s, gids_ctrls_t* c, uint32_t ps, uint64_t off, uint64_t cache_mb,
                                uint64_t num_ele, uint64_t num_ssd) {
  return guarded([&] {
    NEED(s);
    NEED(c);
    s->s.init_controllers(&c->c, ps, off, cache_mb, num_ele, num_ssd);
  });
}

int gids_store_destroy(gids_store_t* s) {
  return guarded([&] { delete s; });
}

int gids_store_set_synchronous(gids_store_t* s, int sync) {
  return guarded([&] {
    NEED(s);
    s->s.synchronous = sync != 0;
  });
}

int gids_store_set_cache_line(gids_store_t* s, uint32_t bytes) {
  return guarded([&] {
    NEED(s);
    s->s.set_cache_line(bytes);
  });
}

int gids_store_set_wait_limit(gids_store_t* s, uint32_t polls) {
  return guarded([&] {
    NEED(s);
    GIDS_CHECK(polls >= 1, GIDS_E_INVAL, "at least one poll");
    s->s.wait_limit = polls;
  });
}

int gids_store_set_cache_policy(gids_store_t* s, int admission, uint32_t ref_max) {
  return guarded([&] {
    NEED(s);
    s->s.set_policy(admission, ref_max);
  });
}

int gids_store_set_gather_blocks(gids_store_t* s, uint32_t max_blocks) {
  return guarded([&] {
    NEED(s);
    s->s.set_gather_blocks(max_blocks);
  });
}

int gids_store_debug_mark_busy(gids_store_t* s, uint64_t line) {
  return guarded([&] {
    NEED(s);
    s->s.debug_mark_busy(line);
  });
}

int gids_store_set_row_layout(gids_store_t* s, uint32_t cache_dim) {
  return guarded([&] {
    NEED(s);
    s->s.set_row_layout(cache_dim);
  });
}

int gids_store_set_sharding(gids_store_t* s, int world, int rank) {
  return guarded([&] {
    NEED(s);
    GIDS_CHECK(world >= 1 && rank >= 0, GIDS_E_INVAL, "bad world/rank");
    s->s.set_sharding((uint32_t)world, (uint32_t)rank);
  });
}

int gids_store_set_replicas(gids_store_t* s, uint64_t max_lines) {
  return guarded([&] {
    NEED(s);
    s->s.set_replicas(max_lines);
  });
}

int gids_store_set_replicated_lines(gids_store_t* s, const uint64_t* lines, uint64_t n) {
  return guarded([&] {
    NEED(s);
    s->s.set_replicated_lines(lines, n);
  });
}

int gids_store_ipc_handle(gids_store_t* s, void* out, size_t len) {
  return guarded([&] {
    NEED(s);
    NEED(out);
    GIDS_CHECK(len >= sizeof(cudaIpcMemHandle_t), GIDS_E_INVAL, "handle buffer must hold 64 bytes");
    s->s.ipc_handle(out);
  });
}

int gids_store_open_peers(gids_store_t* s, const void* handles, int world) {
  return guarded([&] {
    NEED(s);
    NEED(handles);
    GIDS_CHECK(world >= 1, GIDS_E_INVAL, "bad world");
    s->s.open_peers(handles, (uint32_t)world);
  });
}

int gids_store_share_shards(gids_store_t* const* stores, int n) {
  return guarded([&] {
    NEED(stores);
    GIDS_CHECK(n >= 1 && n <= GIDS_MAX_WORLD, GIDS_E_INVAL, "1..8 stores");
    std::vector<gids::Store*> v;
    for (int i = 0; i < n; i++) {
      GIDS_CHECK(stores[i] != nullptr, GIDS_E_INVAL, "null store");
      v.push_back(&stores[i]->s);
    }
    gids::Store::share_in_process(v.data(), (uint32_t)n);
  });
}

int gids_store_peer_copy_gbs(gids_store_t* s, int peer, uint64_t bytes, double* out) {
  return guarded([&] {
    NEED(s);
    NEED(out);
    GIDS_CHECK(peer >= 0, GIDS_E_INVAL, "peer must be >= 0");
    *out = s->s.peer_copy_gbs((uint32_t)peer, bytes);
  });
}

int gids_store_host_read_gbs(gids_store_t* s, uint32_t read_bytes, uint64_t total_bytes, double* out) {
  return guarded([&] {
    NEED(s);
    NEED(out);
    *out = s->s.host_read_gbs(read_bytes, total_bytes);
  });
}

int gids_read_feature(gids_store_t* s, void* out, const int64_t* idx, int64_t n, int dim, int cache_dim,
                      uint64_t key_off, void* stream) {
  return guarded([&] {
    NEED(s);
    GIDS_CHECK(n >= 0, GIDS_E_INVAL, "n must be >= 0");
    void* outs[1] = {out};
    const int64_t* idxs[1] = {idx};
    uint64_t ns[1] = {(uint64_t)n};
    uint64_t ko[1] = {key_off};
    s->s.read_multi(1, outs, idxs, ns, dim, cache_dim, ko, (cudaStream_t)stream);
  });
}

int gids_prefetch(gids_store_t* s, const int64_t* idx, int64_t n, int dim, int cache_dim, uint64_t key_off,
                  void* stream) {
  return guarded([&] {
    NEED(s);
    GIDS_CHECK(n >= 0, GIDS_E_INVAL, "n must be >= 0");
    void* outs[1] = {nullptr};
    const int64_t* idxs[1] = {idx};
    uint64_t ns[1] = {(uint64_t)n};
    uint64_t ko[1] = {key_off};
    s->s.read_multi(1, outs, idxs, ns, dim, cache_dim, ko, (cudaStream_t)stream, true);
  });
}

int gids_read_feature_multi(gids_store_t* s, int k, void* const* outs, const int64_t* const* idxs,
                            const uint64_t* ns, int dim, int cache_dim, const uint64_t* key_offs, void* stream) {
  return guarded([&] {
    NEED(s);
    GIDS_CHECK(k >= 0, GIDS_E_INVAL, "k must be >= 0");
    if (k) {
      NEED(outs);
      NEED(idxs);
      NEED(ns);
    }
    s->s.read_multi(k, outs, idxs, ns, dim, cache_dim, key_offs, (cudaStream_t)stream);
  });
}

int gids_set_window_buffering(gids_store_t* s, const int64_t* idx, int64_t n, int64_t hash_off,
                              uint32_t row_stride_elems, void* stream) {
  return guarded([&] {
    NEED(s);
    s->s.window_buffering(idx, n, hash_off, row_stride_elems, (cudaStream_t)stream);
  });
}

int gids_unset_window_buffering(gids_store_t* s, const int64_t* idx, int64_t n, int64_t hash_off,
                                uint32_t row_stride_elems, void* stream) {
  return guarded([&] {
    NEED(s);
    s->s.window_buffering(idx, n, hash_off, row_stride_elems, (cudaStream_t)stream, gids::WB_UNMARK);
  });
}

int gids_store_pin_rows(gids_store_t* s, const int64_t* idx, int64_t n, int64_t hash_off, uint32_t row_stride_elems,
                        void* stream) {
  return guarded([&] {
    NEED(s);
    s->s.window_buffering(idx, n, hash_off, row_stride_elems, (cudaStream_t)stream, gids::WB_PIN);
  });
}

int gids_store_unpin_rows(gids_store_t* s, const int64_t* idx, int64_t n, int64_t hash_off,
                          uint32_t row_stride_elems, void* stream) {
  return guarded([&] {
    NEED(s);
    s->s.window_buffering(idx, n, hash_off, row_stride_elems, (cudaStream_t)stream, gids::WB_UNPIN);
  });
}

int gids_cpu_backing_buffer(gids_store_t* s, uint64_t dim, uint64_t len) {
  return guarded([&] {
    NEED(s);
    s->s.cpu_backing_buffer(dim, len);
  });
}

int gids_set_cpu_buffer(gids_store_t* s, const int64_t* idx, int num) {
  return guarded([&] {
    NEED(s);
    GIDS_CHECK(num >= 0, GIDS_E_INVAL, "num must be >= 0");
    std::vector<int64_t> h((size_t)num);
    if (num) {
      NEED(idx);
      gids::DeviceGuard g(s->s.device);
      GIDS_CUDA(cudaMemcpy(h.data(), idx, (size_t)num * sizeof(int64_t), cudaMemcpyDefault));
    }
    s->s.set_cpu_buffer(h.data(), num);
  });
}

int gids_set_cpu_buffer_host(gids_store_t* s, const int64_t* idx, int64_t num) {
  return guarded([&] {
    NEED(s);
    s->s.set_cpu_buffer(idx, num);
  });
}

int gids_get_cpu_access_count(gids_store_t* s, uint32_t* out) {
  return guarded([&] {
    NEED(s);
    NEED(out);
    *out = s->s.cpu_access_count();
  });
}

int gids_flush_cpu_access_count(gids_store_t* s) {
  return guarded([&] {
    NEED(s);
    s->s.flush_cpu_access_count();
  });
}

int gids_get_stats(gids_store_t* s, uint64_t* out, int count) {
  return guarded([&] {
    NEED(s);
    NEED(out);
    s->s.get_stats(out, count);
  });
}

int gids_reset_stats(gids_store_t* s) {
  return guarded([&] {
    NEED(s);
    s->s.reset_stats();
  });
}

int gids_print_stats(gids_store_t* s) {
  return guarded([&] {
    NEED(s);
    s->s.print_stats();
  });
}

int gids_get_kernel_time_ms(gids_store_t* s, double* out) {
  return guarded([&] {
    NEED(s);
    NEED(out);
    *out = s->s.kernel_time_ms();
  });
}

int gids_store_synchronize(gids_store_t* s) {
  return guarded([&] {
    NEED(s);
    s->s.synchronize();
  });
}

int gids_store_tensor(gids_store_t* s, const void* src, uint64_t num, uint64_t offset_bytes) {
  return guarded([&] {
    NEED(s);
    s->s.store_tensor(src, num, offset_bytes);
  });
}

int gids_write_range(gids_store_t* s, const void* src, uint64_t nbytes, uint64_t offset_bytes) {
  return guarded([&] {
    NEED(s);
    s->s.write_range(src, nbytes, offset_bytes);
  });
}

int gids_flush_cache(gids_store_t* s) {
  return guarded([&] {
    NEED(s);
    s->s.flush_cache();
  });
}

int gids_read_range_host(gids_store_t* s, void* dst, uint64_t nbytes, uint64_t offset_bytes) {
  return guarded([&] {
    NEED(s);
    GIDS_CHECK(s->s.initialized, GIDS_E_STATE, "read before init_controllers");
    GIDS_CHECK(offset_bytes + nbytes <= s->s.n_pages * (uint64_t)s->s.page_size, GIDS_E_RANGE,
               "read past the end of the range");
    if (nbytes) NEED(dst);
    gids::backing_read(*s->s.ctrls, dst, nbytes, offset_bytes);
  });
}

int gids_fill_synthetic(gids_store_t* s, int kind, uint64_t seed, int threads) {
  return guarded([&] {
    NEED(s);
    GIDS_CHECK(s->s.initialized, GIDS_E_STATE, "fill before init_controllers");
    GIDS_CHECK(gids::synth_elem_bytes(kind) == (int)s->s.elem_bytes, GIDS_E_INVAL,
               "synthetic kind does not match the store's element size");
    gids::DeviceGuard g(s->s.device);
    GIDS_CUDA(cudaDeviceSynchronize());
    gids::backing_fill_synthetic(*s->s.ctrls, kind, seed, threads);
    s->s.flush_cache();
  });
}

int gids_store_geometry(gids_store_t* s, uint64_t* out, int count) {
  return guarded([&] {
    NEED(s);
    NEED(out);
    GIDS_CHECK(s->s.initialized, GIDS_E_STATE, "geometry before init_controllers");
    const uint64_t g[8] = {s->s.n_pages, s->s.ctrls->wrap_pages, s->s.ctrls->ssd.empty() ? 0 : s->s.ctrls->ssd[0].bytes,
                           s->s.n_slots, s->s.page_size,         s->s.ctrls->n_bound,
                           s->s.line_size, s->s.shard_bytes};
    for (int i = 0; i < count && i < 8; i++) out[i] = g[i];
  });
}


int gids_sampler_create(gids_sampler_t** out, int device, const int64_t* indptr, const void* indices, int index_bytes,
                        uint64_t num_nodes, const int* fanouts, int n_layers, uint64_t max_seeds, uint64_t seed) {
  return guarded([&] {
    NEED(out);
    *out = nullptr;
    std::unique_ptr<gids_sampler> h(new gids_sampler());
    h->p = gids::sampler_create(device, indptr, indices, index_bytes, num_nodes, fanouts, n_layers, max_seeds, seed);
    *out = h.release();
  });
}

int gids_sampler_capacity(gids_sampler_t* s, uint64_t* out) {
  return guarded([&] {
    NEED(s);
    NEED(out);
    *out = gids::sampler_capacity(s->p);
  });
}

int gids_sampler_sample(gids_sampler_t* s, const int64_t* seeds, uint64_t n_seeds, int64_t* out_nodes,
                        uint64_t out_cap, uint64_t* count_dev, uint64_t* count_host, int64_t call, void* stream) {
  return guarded([&] {
    NEED(s);
    gids::sampler_sample(s->p, seeds, n_seeds, out_nodes, out_cap, count_dev, count_host, call, (cudaStream_t)stream);
  });
}

int gids_sampler_destroy(gids_sampler_t* s) {
  return guarded([&] { delete s; });
}

int gids_pagerank(int device, const int64_t* indptr, const void* indices, int index_bytes, uint64_t num_nodes,
                  int iters, double damping, float* pv, uint64_t* order_keys, void* stream) {
  return guarded([&] {
    gids::pagerank(device, indptr, indices, index_bytes, num_nodes, iters, damping, pv, order_keys,
                   (cudaStream_t)stream);
  });
}

int gids_out_degree(int device, const void* indices, int index_bytes, uint64_t num_edges, uint64_t num_nodes,
                    uint32_t* counts, void* stream) {
  return guarded([&] {
    gids::out_degree(device, indices, index_bytes, num_edges, num_nodes, counts, (cudaStream_t)stream);
  });
}

}  // extern "C"
