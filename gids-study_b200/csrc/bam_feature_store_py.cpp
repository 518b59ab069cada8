// pybind11 module BAM_Feature_Store: the reference's Python boundary
// (gids_module/gids_nvme.cu:823-893) rebuilt over the C ABI of libgids_b200.
// Class and method names, argument order and meaning follow the reference;
// every method releases the GIL and raises RuntimeError on failure. Methods
// marked "extension" have no reference counterpart.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "gids_b200.h"

namespace py = pybind11;

namespace {

void check(int rc) {
  if (rc != GIDS_OK) {
    char buf[1024];
    gids_last_error(buf, sizeof(buf));
    throw std::runtime_error(std::string("gids: ") + gids_strerror(rc) + ": " + buf);
  }
}

struct Controllers {
  gids_ctrls_t* c = nullptr;
  uint32_t n_ctrls = 0;
  Controllers() { check(gids_ctrls_create(&c)); }
  ~Controllers() {
    if (c) gids_ctrls_destroy(c);
  }
  Controllers(const Controllers&) = delete;
  // GIDS_Controllers::init_GIDS_controllers (gids_nvme.cu:93-107)
  void init(uint32_t n, uint64_t q_depth, uint64_t n_queues, const std::vector<int>& ssd_list) {
    std::vector<int32_t> l(ssd_list.begin(), ssd_list.end());
    if (l.size() < n) throw std::runtime_error("ssd_list shorter than the number of controllers");
    check(gids_ctrls_init(c, n, q_depth, n_queues, l.data()));
    n_ctrls = n;
  }
  // extension: emulated-SSD capacity (bytes per SSD, 0 = whole stripe) and file pattern
  void set_emulation(uint64_t capacity, const std::string& pattern) {
    check(gids_ctrls_set_emulation(c, capacity, pattern.c_str()));
  }
  // extension: the backing store without a GPU cache
  void bind(uint32_t num_ssd, uint32_t page_size, uint64_t read_off_pages, uint64_t range_bytes) {
    check(gids_ctrls_bind(c, num_ssd, page_size, read_off_pages, range_bytes));
  }
  void write(uint64_t src, uint64_t nbytes, uint64_t off) { check(gids_ctrls_write(c, (const void*)src, nbytes, off)); }
  void read_into(uint64_t dst, uint64_t nbytes, uint64_t off) { check(gids_ctrls_read(c, (void*)dst, nbytes, off)); }
  void fill_synthetic(int kind, uint64_t seed, int threads) { check(gids_ctrls_fill_synthetic(c, kind, seed, threads)); }
  py::dict geometry() {
    uint64_t g[4] = {0};
    check(gids_ctrls_geometry(c, g, 4));
    py::dict d;
    d["range_pages"] = g[0];
    d["wrap_pages"] = g[1];
    d["ssd_bytes"] = g[2];
    d["num_ssd"] = g[3];
    return d;
  }
};

class FeatureStore {
 public:
  explicit FeatureStore(uint32_t eb) : eb_(eb) {}
  ~FeatureStore() {
    if (s_) gids_store_destroy(s_);
  }
  FeatureStore(const FeatureStore&) = delete;

  gids_store_t* s() const {
    if (!s_) throw std::runtime_error("gids: init_controllers has not been called");
    return s_;
  }
  // extension: device for the store (default: the current CUDA device at init_controllers)
  void set_device(int d) {
    if (s_) throw std::runtime_error("gids: set_device after init_controllers");
    device_ = d;
  }
  // BAM_Feature_Store<T>::init_controllers (gids_nvme.cu:166-221)
  void init_controllers(Controllers& ctrl, uint32_t ps, uint64_t read_off, uint64_t cache_size, uint64_t num_ele,
                        uint64_t num_ssd) {
    if (s_) throw std::runtime_error("gids: init_controllers called twice");
    int dev = device_;
    if (dev < 0) check(gids_current_device(&dev));
    gids_store_t* s = nullptr;
    check(gids_store_create(&s, eb_, dev));
    int rc = GIDS_OK;
    if (world_ > 1) rc = gids_store_set_sharding(s, world_, rank_);
    if (rc == GIDS_OK && line_) rc = gids_store_set_cache_line(s, line_);
    if (rc == GIDS_OK && rep_max_) rc = gids_store_set_replicas(s, rep_max_);
    if (rc == GIDS_OK) rc = gids_store_init_controllers(s, ctrl.c, ps, read_off, cache_size, num_ele, num_ssd);
    if (rc != GIDS_OK) {
      char buf[1024];
      gids_last_error(buf, sizeof(buf));
      gids_store_destroy(s);
      throw std::runtime_error(std::string("gids: ") + gids_strerror(rc) + ": " + buf);
    }
    s_ = s;
    page_size_ = ps;
  }
  // read_feature (gids_nvme.cu:324-364)
  void read_feature(uint64_t out, uint64_t idx, int64_t n, int dim, int cache_dim, uint64_t key_off,
                    uint64_t stream) {
    check(gids_read_feature(s(), (void*)out, (const int64_t*)idx, n, dim, cache_dim, key_off, (void*)stream));
  }
  // read_feature_hetero / read_feature_merged_hetero (gids_nvme.cu:382-445, 531-593)
  void read_hetero(int k, const std::vector<uint64_t>& outs, const std::vector<uint64_t>& idxs,
                   const std::vector<uint64_t>& ns, int dim, int cache_dim, const std::vector<uint64_t>& key_off,
                   uint64_t stream) {
    check_lists(k, outs, idxs, ns);
    if (key_off.size() < (size_t)k) throw std::runtime_error("gids: key_off list shorter than k");
    check(gids_read_feature_multi(s(), k, (void* const*)outs.data(), (const int64_t* const*)idxs.data(), ns.data(),
                                  dim, cache_dim, key_off.data(), (void*)stream));
  }
  // read_feature_merged (gids_nvme.cu:456-518)
  void read_merged(int k, const std::vector<uint64_t>& outs, const std::vector<uint64_t>& idxs,
                   const std::vector<uint64_t>& ns, int dim, int cache_dim, uint64_t stream) {
    check_lists(k, outs, idxs, ns);
    check(gids_read_feature_multi(s(), k, (void* const*)outs.data(), (const int64_t* const*)idxs.data(), ns.data(),
                                  dim, cache_dim, nullptr, (void*)stream));
  }
  // set_window_buffering (gids_nvme.cu:242-249)
  void set_window_buffering(uint64_t idx, int64_t n, int64_t hash_off, uint64_t stream) {
    check(gids_set_window_buffering(s(), (const int64_t*)idx, n, hash_off, 0, (void*)stream));
  }
  // extension: take back the marks of a window that will not be gathered
  void unset_window_buffering(uint64_t idx, int64_t n, int64_t hash_off, uint64_t stream) {
    check(gids_unset_window_buffering(s(), (const int64_t*)idx, n, hash_off, 0, (void*)stream));
  }
  // extension: window-buffer prefetch, the rows' lines brought into the cache without an output
  void prefetch(uint64_t idx, int64_t n, int dim, int cache_dim, int64_t key_off, uint64_t stream) {
    check(gids_prefetch(s(), (const int64_t*)idx, n, dim, cache_dim, (uint64_t)key_off, (void*)stream));
  }
  // extension: permanent pins of the rows' cache lines (a static hot set)
  void pin_rows(uint64_t idx, int64_t n, int64_t hash_off, uint64_t stream) {
    check(gids_store_pin_rows(s(), (const int64_t*)idx, n, hash_off, 0, (void*)stream));
  }
  void unpin_rows(uint64_t idx, int64_t n, int64_t hash_off, uint64_t stream) {
    check(gids_store_unpin_rows(s(), (const int64_t*)idx, n, hash_off, 0, (void*)stream));
  }
  // cpu_backing_buffer (gids_nvme.cu:123-139)
  void cpu_backing_buffer(uint64_t dim, uint64_t len) { check(gids_cpu_backing_buffer(s(), dim, len)); }
  // set_cpu_buffer (gids_nvme.cu:694-711)
  void set_cpu_buffer(uint64_t idx, int num) { check(gids_set_cpu_buffer(s(), (const int64_t*)idx, num)); }
  // flush_cache (gids_nvme.cu:673-677)
  void flush_cache() { check(gids_flush_cache(s())); }
  // store_tensor (gids_nvme.cu:616-663)
  void store_tensor(uint64_t ptr, uint64_t num, uint64_t offset) {
    check(gids_store_tensor(s(), (const void*)ptr, num, offset));
  }
  // read_tensor (gids_nvme.cu:764-770): prints num elements from element offset
  void read_tensor(uint64_t num, uint64_t offset) {
    std::vector<char> buf(num * eb_);
    check(gids_read_range_host(s(), buf.data(), buf.size(), offset * eb_));
    printf("offset:%llu\n", (unsigned long long)offset);
    for (uint64_t i = 0; i < num; i++) {
      if (eb_ == 4) {
        float v;
        memcpy(&v, buf.data() + i * 4, 4);
        printf("read data: %f\n", v);
      } else if (eb_ == 8) {
        long long v;
        memcpy(&v, buf.data() + i * 8, 8);
        printf("read data: %lld\n", v);
      } else {
        uint16_t v;
        memcpy(&v, buf.data() + i * 2, 2);
        printf("read data: 0x%04x\n", v);
      }
    }
    fflush(stdout);
  }
  // get_cpu_access_count / flush_cpu_access_count (gids_nvme.cu:779-794)
  uint32_t get_cpu_access_count() {
    uint32_t v = 0;
    check(gids_get_cpu_access_count(s(), &v));
    return v;
  }
  void flush_cpu_access_count() { check(gids_flush_cpu_access_count(s())); }
  // print_stats (gids_nvme.cu:279-300)
  void print_stats() { check(gids_print_stats(s())); }
  // set_offsets / get_offset_array (gids_nvme.cu:721-748): host triple used by
  // the graph-on-SSD sampler, kept for interface compatibility
  void set_offsets(uint64_t a, uint64_t b, uint64_t c) { offsets_ = {a, b, c}; }
  uint64_t get_offset_array() { return (uint64_t)(uintptr_t)offsets_.data(); }

  // ---- extensions
  // sharded cache (must be set before init_controllers)
  void set_sharding(int world, int rank) {
    if (s_) throw std::runtime_error("gids: set_sharding after init_controllers");
    world_ = world;
    rank_ = rank;
  }
  // replicated lines: entries reserved before init_controllers, then the set
  // (host int64 array of strictly increasing cache-line ids)
  void set_replicas(uint64_t max_lines) {
    if (s_) throw std::runtime_error("gids: set_replicas after init_controllers");
    rep_max_ = max_lines;
  }
  void set_replicated_lines(uint64_t lines_ptr, uint64_t n) {
    check(gids_store_set_replicated_lines(s(), (const uint64_t*)lines_ptr, n));
  }
  // cache line in bytes (must be set before init_controllers; 0 = the page)
  void set_cache_line(uint32_t bytes) {
    if (s_) throw std::runtime_error("gids: set_cache_line after init_controllers");
    line_ = bytes;
  }
  // replacement policy: admission on the second miss, clock counter ceiling
  void set_cache_policy(int admission, uint32_t ref_max) { check(gids_store_set_cache_policy(s(), admission, ref_max)); }
  // cap on the gather's grid (0: every resident block)
  void set_gather_blocks(uint32_t n) { check(gids_store_set_gather_blocks(s(), n)); }
  // NVLink bandwidth: a timed copy from a peer rank's shard (GB/s)
  double peer_copy_gbs(int peer, uint64_t bytes) {
    double v = 0.0;
    check(gids_store_peer_copy_gbs(s(), peer, bytes, &v));
    return v;
  }
  // host-link bandwidth of random reads at the gather's access size (GB/s)
  double host_read_gbs(uint32_t read_bytes, uint64_t total_bytes) {
    double v = 0.0;
    check(gids_store_host_read_gbs(s(), read_bytes, total_bytes, &v));
    return v;
  }
  py::bytes ipc_handle() {
    char h[64];
    check(gids_store_ipc_handle(s(), h, sizeof(h)));
    return py::bytes(h, sizeof(h));
  }
  void open_peers(const std::vector<std::string>& handles) {
    std::string all;
    for (const auto& h : handles) {
      if (h.size() != 64) throw std::runtime_error("gids: IPC handles are 64 bytes");
      all += h;
    }
    py::gil_scoped_release r;
    check(gids_store_open_peers(s(), all.data(), (int)handles.size()));
  }
  void set_synchronous(bool v) { check(gids_store_set_synchronous(s(), v ? 1 : 0)); }
  void set_row_layout(uint32_t cache_dim) { check(gids_store_set_row_layout(s(), cache_dim)); }
  void synchronize() { check(gids_store_synchronize(s())); }
  py::dict get_stats() {
    uint64_t v[GIDS_STAT_COUNT] = {0};
    {
      py::gil_scoped_release r;
      check(gids_get_stats(s(), v, GIDS_STAT_COUNT));
    }
    py::dict d;
    static const char* names[] = {"access",      "hit",       "miss",          "read_io",     "bypass",
                                  "cpu_rows",    "rows",      "wait_timeouts", "bad_ids",     "bytes_hit",
                                  "bytes_miss",  "bytes_bypass", "bytes_cpu",   "evictions",   "launches",
                                  "bytes_peer",  "ns_lookup", "ns_fill_wait",  "ns_copy",     "ns_release",
                                  "prefetched"};
    static_assert(sizeof(names) / sizeof(names[0]) == GIDS_STAT_COUNT, "one name per counter");
    for (int i = 0; i < GIDS_STAT_COUNT; i++) d[names[i]] = v[i];
    return d;
  }
  void reset_stats() { check(gids_reset_stats(s())); }
  double kernel_time_ms() {
    double v = 0;
    check(gids_get_kernel_time_ms(s(), &v));
    return v;
  }
  void fill_synthetic(int kind, uint64_t seed, int threads) { check(gids_fill_synthetic(s(), kind, seed, threads)); }
  void write_range(uint64_t ptr, uint64_t nbytes, uint64_t offset) {
    check(gids_write_range(s(), (const void*)ptr, nbytes, offset));
  }
  void read_range_into(uint64_t dst, uint64_t nbytes, uint64_t offset) {
    check(gids_read_range_host(s(), (void*)dst, nbytes, offset));
  }
  py::dict geometry() {
    uint64_t g[8] = {0};
    check(gids_store_geometry(s(), g, 8));
    py::dict d;
    d["range_pages"] = g[0];
    d["wrap_pages"] = g[1];
    d["ssd_bytes"] = g[2];
    d["cache_slots"] = g[3];
    d["page_size"] = g[4];
    d["num_ssd"] = g[5];
    d["cache_line"] = g[6];
    d["shard_bytes"] = g[7];
    return d;
  }
  uint32_t elem_bytes() const { return eb_; }
  uint64_t handle() const { return (uint64_t)(uintptr_t)s(); }

 private:
  static void check_lists(int k, const std::vector<uint64_t>& o, const std::vector<uint64_t>& i,
                          const std::vector<uint64_t>& n) {
    if (k < 0 || o.size() < (size_t)k || i.size() < (size_t)k || n.size() < (size_t)k)
      throw std::runtime_error("gids: pointer lists shorter than k");
  }
  uint32_t eb_;
  int device_ = -1;
  int world_ = 1, rank_ = 0;
  uint32_t line_ = 0;
  uint64_t rep_max_ = 0;
  uint32_t page_size_ = 0;
  gids_store_t* s_ = nullptr;
  std::vector<uint64_t> offsets_{0, 0, 0};
};

template <uint32_t EB, int TAG>
struct TypedStore : FeatureStore {
  TypedStore() : FeatureStore(EB) {}
};

template <uint32_t EB, int TAG>
void bind_store(py::module_& m, const char* name) {
  using S = TypedStore<EB, TAG>;
  using R = py::call_guard<py::gil_scoped_release>;
  py::class_<S>(m, name)
      .def(py::init<>())
      .def("init_controllers", &S::init_controllers, py::arg("ctrl"), py::arg("ps"), py::arg("read_off"),
           py::arg("cache_size"), py::arg("num_ele"), py::arg("num_ssd") = 1, R())
      .def("read_feature", &S::read_feature, py::arg("i_ptr"), py::arg("i_index_ptr"), py::arg("num_index"),
           py::arg("dim"), py::arg("cache_dim"), py::arg("key_off") = 0, py::arg("stream") = 0, R())
      .def("read_feature_hetero", &S::read_hetero, py::arg("num_iter"), py::arg("i_ptr_list"),
           py::arg("i_index_ptr_list"), py::arg("num_index"), py::arg("dim"), py::arg("cache_dim"),
           py::arg("key_off"), py::arg("stream") = 0, R())
      .def("read_feature_merged_hetero", &S::read_hetero, py::arg("num_iter"), py::arg("i_ptr_list"),
           py::arg("i_index_ptr_list"), py::arg("num_index"), py::arg("dim"), py::arg("cache_dim"),
           py::arg("key_off"), py::arg("stream") = 0, R())
      .def("read_feature_merged", &S::read_merged, py::arg("num_iter"), py::arg("i_ptr_list"),
           py::arg("i_index_ptr_list"), py::arg("num_index"), py::arg("dim"), py::arg("cache_dim") = 1024,
           py::arg("stream") = 0, R())
      .def("set_window_buffering", &S::set_window_buffering, py::arg("id_idx"), py::arg("num_pages"),
           py::arg("hash_off") = 0, py::arg("stream") = 0, R())
      .def("unset_window_buffering", &S::unset_window_buffering, py::arg("id_idx"), py::arg("num_pages"),
           py::arg("hash_off") = 0, py::arg("stream") = 0, R())
      .def("prefetch", &S::prefetch, py::arg("i_index_ptr"), py::arg("num_index"), py::arg("dim"),
           py::arg("cache_dim") = 1024, py::arg("key_off") = 0, py::arg("stream") = 0, R())
      .def("pin_rows", &S::pin_rows, py::arg("id_idx"), py::arg("num"), py::arg("hash_off") = 0,
           py::arg("stream") = 0, R())
      .def("unpin_rows", &S::unpin_rows, py::arg("id_idx"), py::arg("num"), py::arg("hash_off") = 0,
           py::arg("stream") = 0, R())
      .def("cpu_backing_buffer", &S::cpu_backing_buffer, py::arg("dim"), py::arg("len"), R())
      .def("set_cpu_buffer", &S::set_cpu_buffer, py::arg("idx_buffer"), py::arg("num"), R())
      .def("flush_cache", &S::flush_cache, R())
      .def("store_tensor", &S::store_tensor, py::arg("tensor_ptr"), py::arg("num"), py::arg("offset"), R())
      .def("read_tensor", &S::read_tensor, py::arg("num"), py::arg("offset"), R())
      .def("get_array_ptr",
           [](S&) -> uint64_t {
             throw std::runtime_error(
                 "gids: get_array_ptr exposes the BaM device array used by graph-structure sampling, "
                 "which this library does not implement");
           })
      .def("get_offset_array", &S::get_offset_array)
      .def("set_offsets", &S::set_offsets)
      .def("get_cpu_access_count", &S::get_cpu_access_count, R())
      .def("flush_cpu_access_count", &S::flush_cpu_access_count, R())
      .def("print_stats", &S::print_stats, R())
      // extensions
      .def("set_device", &S::set_device)
      .def("set_sharding", &S::set_sharding, py::arg("world"), py::arg("rank"))
      .def("set_replicas", &S::set_replicas, py::arg("max_lines"))
      .def("set_replicated_lines", &S::set_replicated_lines, py::arg("lines_ptr"), py::arg("n"), R())
      .def("set_cache_line", &S::set_cache_line, py::arg("bytes"))
      .def("set_cache_policy", &S::set_cache_policy, py::arg("admission"), py::arg("ref_max"))
      .def("set_gather_blocks", &S::set_gather_blocks, py::arg("max_blocks"))
      .def("ipc_handle", &S::ipc_handle)
      .def("peer_copy_gbs", &S::peer_copy_gbs, py::arg("peer"), py::arg("bytes"), R())
      .def("host_read_gbs", &S::host_read_gbs, py::arg("read_bytes"), py::arg("total_bytes"), R())
      .def("open_peers", &S::open_peers)
      .def("set_synchronous", &S::set_synchronous, R())
      .def("set_row_layout", &S::set_row_layout, R())
      .def("synchronize", &S::synchronize, R())
      .def("get_stats", &S::get_stats)
      .def("reset_stats", &S::reset_stats, R())
      .def("kernel_time_ms", &S::kernel_time_ms, R())
      .def("fill_synthetic", &S::fill_synthetic, py::arg("kind"), py::arg("seed"), py::arg("threads") = 0, R())
      .def("write_range", &S::write_range, R())
      .def("read_range_into", &S::read_range_into, R())
      .def("geometry", &S::geometry)
      .def_property_readonly("elem_bytes", &S::elem_bytes)
      .def_property_readonly("handle", &S::handle);
}

}  // namespace

// extension: the GPU neighbour sampler over a CSC graph (gids_sampler_*)
class Sampler {
 public:
  Sampler(int device, uint64_t indptr, uint64_t indices, int index_bytes, uint64_t num_nodes,
          const std::vector<int>& fanouts, uint64_t max_seeds, uint64_t seed) {
    check(gids_sampler_create(&s_, device, (const int64_t*)indptr, (const void*)indices, index_bytes, num_nodes,
                              fanouts.data(), (int)fanouts.size(), max_seeds, seed));
  }
  ~Sampler() {
    if (s_) gids_sampler_destroy(s_);
  }
  uint64_t capacity() {
    uint64_t v = 0;
    check(gids_sampler_capacity(s_, &v));
    return v;
  }
  // returns the node count (waits for the stream) unless count_dev is given
  uint64_t sample(uint64_t seeds, uint64_t n_seeds, uint64_t out, uint64_t out_cap, uint64_t count_dev, int64_t call,
                  uint64_t stream) {
    uint64_t host = 0;
    check(gids_sampler_sample(s_, (const int64_t*)seeds, n_seeds, (int64_t*)out, out_cap, (uint64_t*)count_dev,
                              count_dev ? nullptr : &host, call, (void*)stream));
    return host;
  }

 private:
  gids_sampler_t* s_ = nullptr;
};

PYBIND11_MODULE(BAM_Feature_Store, m) {
  m.doc() = "B200 GIDS feature store (drop-in for the reference's BAM_Feature_Store pybind module)";
  py::class_<Controllers>(m, "GIDS_Controllers")
      .def(py::init<>())
      .def("init_GIDS_controllers", &Controllers::init, py::arg("num_ctrls"), py::arg("q_depth"), py::arg("num_q"),
           py::arg("ssd_list"))
      .def("set_emulation", &Controllers::set_emulation, py::arg("capacity_bytes_per_ssd") = 0,
           py::arg("path_pattern") = std::string())
      .def("bind", &Controllers::bind, py::arg("num_ssd"), py::arg("page_size"), py::arg("read_off_pages"),
           py::arg("range_bytes"), py::call_guard<py::gil_scoped_release>())
      .def("write", &Controllers::write, py::call_guard<py::gil_scoped_release>())
      .def("read_into", &Controllers::read_into, py::call_guard<py::gil_scoped_release>())
      .def("fill_synthetic", &Controllers::fill_synthetic, py::arg("kind"), py::arg("seed"), py::arg("threads") = 0,
           py::call_guard<py::gil_scoped_release>())
      .def("geometry", &Controllers::geometry)
      .def_readonly("n_ctrls", &Controllers::n_ctrls);
  bind_store<4, 0>(m, "BAM_Feature_Store_float");
  bind_store<8, 0>(m, "BAM_Feature_Store_long");
  bind_store<2, 0>(m, "BAM_Feature_Store_half");
  bind_store<2, 1>(m, "BAM_Feature_Store_bfloat16");
  m.def("version", []() { return std::string(gids_version()); });
  py::class_<Sampler>(m, "GIDS_Sampler")
      .def(py::init<int, uint64_t, uint64_t, int, uint64_t, const std::vector<int>&, uint64_t, uint64_t>(),
           py::arg("device"), py::arg("indptr"), py::arg("indices"), py::arg("index_bytes"), py::arg("num_nodes"),
           py::arg("fanouts"), py::arg("max_seeds"), py::arg("seed"))
      .def("capacity", &Sampler::capacity)
      .def("sample", &Sampler::sample, py::arg("seeds"), py::arg("n_seeds"), py::arg("out"), py::arg("out_cap"),
           py::arg("count_dev") = 0, py::arg("call") = -1, py::arg("stream") = 0,
           py::call_guard<py::gil_scoped_release>());
  // extension: out-degree histogram of a CSC graph (gids_out_degree)
  m.def(
      "out_degree",
      [](int device, uint64_t indices, int index_bytes, uint64_t num_edges, uint64_t num_nodes, uint64_t counts,
         uint64_t stream) {
        check(gids_out_degree(device, (const void*)indices, index_bytes, num_edges, num_nodes, (uint32_t*)counts,
                              (void*)stream));
      },
      py::arg("device"), py::arg("indices"), py::arg("index_bytes"), py::arg("num_edges"), py::arg("num_nodes"),
      py::arg("counts"), py::arg("stream") = 0, py::call_guard<py::gil_scoped_release>());
  // extension: compute_pagerank of the pin-list generator in float32 (gids_pagerank)
  m.def(
      "pagerank",
      [](int device, uint64_t indptr, uint64_t indices, int index_bytes, uint64_t n, int iters, double damping,
         uint64_t pv, uint64_t keys, uint64_t stream) {
        check(gids_pagerank(device, (const int64_t*)indptr, (const void*)indices, index_bytes, n, iters, damping,
                            (float*)pv, (uint64_t*)keys, (void*)stream));
      },
      py::arg("device"), py::arg("indptr"), py::arg("indices"), py::arg("index_bytes"), py::arg("num_nodes"),
      py::arg("iters"), py::arg("damping"), py::arg("pv"), py::arg("keys") = 0, py::arg("stream") = 0,
      py::call_guard<py::gil_scoped_release>());
  // extension: one process driving every GPU of a sharded cache
  m.def("share_shards", [](py::list stores) {
    std::vector<gids_store_t*> v;
    for (auto h : stores) v.push_back((gids_store_t*)(uintptr_t)h.attr("handle").cast<uint64_t>());
    py::gil_scoped_release r;
    check(gids_store_share_shards(v.data(), (int)v.size()));
  });
}
