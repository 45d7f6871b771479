// pybind11 module `flashtrie`: the reference's Python surface
// (tools/bindings.cpp:24-122) on top of the libftcore C ABI.
//
// Same names, keyword arguments, defaults and return shapes:
//   Trie(), .load, .mmap, .build(token_rows), .total_size, .num_tries,
//   .num_keys, .num_nodes, .save, .clear,
//   .init_tbs_gpu(max_batch_size, max_num_topk=1024, max_num_outpos=64,
//                 max_num_out_beams=8192, max_num_out_tokens=8192*64,
//                 max_num_inter_beams=1024*1024, radix_topk_threshold=1024)
//   tbs(trie, beams, topk_id, topk_logp, token_logp_threshold,
//       sents_logp_threshold, length_norm, early_exit, use_gpu=False)
//       -> (out_sent, out_logp_norm, ms)
//   bs_tbs_gpu(trie, batch_size, batch_beams, batch_topk_id, batch_topk_logp,
//       token_logp_threshold, sents_logp_threshold, length_norm, early_exit)
//       -> (batch_out_sent, batch_out_logp_norm, ms, phase_times)
//   load_topk_keys_and_scores(dataset_dir) -> (keys, scores)
// Lists of lists are accepted as in the reference; numpy arrays of matching
// shape are read without per-element conversion.  Every search runs on the
// B200 engine (`use_gpu` is accepted for signature compatibility).
// Extension: keyword-only return_key_ids=True appends the key id of every
// result beam (LoudsTrie::lookup's id, louds-trie.cc:56-72) to the returned
// tuple: tbs -> (..., ms, key_ids), bs_tbs_gpu -> (..., phase_times, key_ids).
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cfloat>
#include <chrono>
#include <cstdint>
#include <fstream>
#include <iostream>
#include <limits>
#include <memory>
#include <numeric>
#include <sstream>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "../../../include/flashtrie_b200.h"

namespace py = pybind11;

namespace {

void check(int rc) {
  if (rc == FT_OK) return;
  const std::string msg = ft_last_error();
  if (rc == FT_ERR_INVALID_ARG) throw py::value_error(msg);
  throw std::runtime_error(msg);  // marisa::Exception surfaces as RuntimeError too
}

class PyTrie {
 public:
  PyTrie() { check(ft_trie_create(&h_)); }
  ~PyTrie() { ft_trie_destroy(h_); }
  PyTrie(const PyTrie &) = delete;
  PyTrie &operator=(const PyTrie &) = delete;
  ft_trie *h() const { return h_; }

  void load(const std::string &path) { check(ft_trie_load(h_, path.c_str())); }
  void mmap(const std::string &path) { check(ft_trie_mmap(h_, path.c_str())); }
  void save(const std::string &path) const { check(ft_trie_save(h_, path.c_str())); }
  void clear() { check(ft_trie_clear(h_)); }
  ft_trie_info info() const {
    ft_trie_info i;
    check(ft_trie_get_info(h_, &i));
    return i;
  }
  void build(py::object rows);
  void init_tbs_gpu(uint64_t max_batch, uint64_t topk, uint64_t outpos, uint64_t out_beams, uint64_t out_tokens,
                    uint64_t inter_beams, uint64_t radix) {
    py::gil_scoped_release nogil;
    check(ft_trie_init_tbs_gpu(h_, max_batch, topk, outpos, out_beams, out_tokens, inter_beams, radix));
  }
  uint64_t max_batch() const {
    uint64_t m = 0;
    check(ft_trie_get_max_batch_size(h_, &m));
    return m;
  }

 private:
  ft_trie *h_ = nullptr;
};

// ------------------------------------------------------------ converters
uint32_t to_label(PyObject *o) {
  unsigned long long v = PyLong_AsUnsignedLongLong(o);
  if (v == (unsigned long long)-1 && PyErr_Occurred()) {
    PyErr_Clear();
    throw py::type_error("token ids must be integers in [0, 2^32)");
  }
  if (v > 0xFFFFFFFFull) throw py::type_error("token ids must be integers in [0, 2^32)");
  return (uint32_t)v;
}

float to_float(PyObject *o) {
  const double d = PyFloat_AsDouble(o);
  if (d == -1.0 && PyErr_Occurred()) {
    PyErr_Clear();
    throw py::type_error("log-probabilities must be numbers");
  }
  return (float)d;
}

// Appends a 1-D sequence of labels to `out`; returns its length.
size_t append_labels(py::handle seq, std::vector<uint32_t> &out) {
  if (py::isinstance<py::array>(seq)) {
    auto a = py::array_t<uint32_t, py::array::c_style | py::array::forcecast>::ensure(seq);
    if (!a || a.ndim() != 1) throw py::type_error("expected a 1-D sequence of token ids");
    out.insert(out.end(), a.data(), a.data() + a.size());
    return (size_t)a.size();
  }
  PyObject *fast = PySequence_Fast(seq.ptr(), "expected a sequence of token ids");
  if (!fast) throw py::error_already_set();
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fast);
  PyObject **items = PySequence_Fast_ITEMS(fast);
  try {
    for (Py_ssize_t i = 0; i < n; ++i) out.push_back(to_label(items[i]));
  } catch (...) {
    Py_DECREF(fast);
    throw;
  }
  Py_DECREF(fast);
  return (size_t)n;
}

size_t append_floats(py::handle seq, std::vector<float> &out) {
  if (py::isinstance<py::array>(seq)) {
    auto a = py::array_t<float, py::array::c_style | py::array::forcecast>::ensure(seq);
    if (!a || a.ndim() != 1) throw py::type_error("expected a 1-D sequence of log-probabilities");
    out.insert(out.end(), a.data(), a.data() + a.size());
    return (size_t)a.size();
  }
  PyObject *fast = PySequence_Fast(seq.ptr(), "expected a sequence of log-probabilities");
  if (!fast) throw py::error_already_set();
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(fast);
  PyObject **items = PySequence_Fast_ITEMS(fast);
  try {
    for (Py_ssize_t i = 0; i < n; ++i) out.push_back(to_float(items[i]));
  } catch (...) {
    Py_DECREF(fast);
    throw;
  }
  Py_DECREF(fast);
  return (size_t)n;
}

void PyTrie::build(py::object rows) {
  std::vector<uint32_t> tokens;
  std::vector<uint64_t> offsets{0};
  if (py::isinstance<py::array>(rows)) {
    auto a = py::array_t<uint32_t, py::array::c_style | py::array::forcecast>::ensure(rows);
    if (!a || a.ndim() != 2) throw py::type_error("token_rows: expected a list of token lists or a 2-D array");
    const size_t R = (size_t)a.shape(0), C = (size_t)a.shape(1);
    tokens.assign(a.data(), a.data() + R * C);
    for (size_t r = 0; r < R; ++r) offsets.push_back((r + 1) * C);
  } else {
    for (py::handle row : rows) {
      append_labels(row, tokens);
      offsets.push_back(tokens.size());
    }
  }
  py::gil_scoped_release nogil;
  check(ft_trie_build(h_, tokens.data(), offsets.data(), offsets.size() - 1));
}

// One request as contiguous buffers: numpy rows of the right dtype and
// layout are borrowed (the array objects are kept alive here), lists are
// converted into owned vectors.
struct Req {
  std::vector<uint32_t> beams;
  std::vector<uint32_t> ids_own;
  std::vector<float> lp_own;
  py::object ids_keep, lp_keep;
  const uint32_t *ids = nullptr;
  const float *lp = nullptr;
  uint32_t L = 0, K = 0;
};

void convert_request(py::handle beams, py::handle topk_id, py::handle topk_logp, Req &r) {
  append_labels(beams, r.beams);
  r.L = (uint32_t)r.beams.size();
  if (py::isinstance<py::array>(topk_id) && py::isinstance<py::array>(topk_logp)) {
    auto ai = py::array_t<uint32_t, py::array::c_style | py::array::forcecast>::ensure(topk_id);
    auto al = py::array_t<float, py::array::c_style | py::array::forcecast>::ensure(topk_logp);
    if (!ai || !al || ai.ndim() != 2 || al.ndim() != 2 || ai.shape(0) != al.shape(0) || ai.shape(1) != al.shape(1))
      throw py::value_error("topk_id and topk_logp must be 2-D arrays of the same shape");
    if ((uint32_t)ai.shape(0) != r.L) throw py::value_error("topk_id must have one row per entry of beams");
    r.K = (uint32_t)ai.shape(1);
    r.ids = ai.data();
    r.lp = al.data();
    r.ids_keep = std::move(ai);
    r.lp_keep = std::move(al);
    return;
  }
  size_t rows_i = 0, rows_l = 0;
  bool first = true;
  for (py::handle row : topk_id) {
    const size_t k = append_labels(row, r.ids_own);
    if (first) r.K = (uint32_t)k;
    else if (k != r.K) throw py::value_error("all topk_id rows must have the same length");
    first = false;
    ++rows_i;
  }
  for (py::handle row : topk_logp) {
    const size_t k = append_floats(row, r.lp_own);
    if (k != r.K) throw py::value_error("topk_logp rows must match the topk_id rows");
    ++rows_l;
  }
  if (rows_i != r.L || rows_l != r.L) throw py::value_error("topk_id and topk_logp must have one row per entry of beams");
  r.ids = r.ids_own.data();
  r.lp = r.lp_own.data();
}

double msec_truncated(std::chrono::high_resolution_clock::time_point a, std::chrono::high_resolution_clock::time_point b) {
  // Same rounding as the reference (include/marisa/tbs_input.h:28-34).
  const double ms = 1000.0 * std::chrono::duration<double>(b - a).count();
  return (double)(int)(100 * ms) / 100.;
}

struct Out {
  std::vector<double> lpn;
  std::vector<uint32_t> len;
  std::vector<uint32_t> key;  // key ids, when asked for
  std::unique_ptr<uint32_t[]> tok;  // cap * stride slots, only the first len[b] of beam b are written
  ft_result res;
};

void prepare_out(const Req &r, Out &o, bool keys) {
  const uint32_t cap = std::max<uint32_t>(r.L ? r.beams[r.L - 1] : 0, 1);
  const uint32_t stride = std::max<uint32_t>(r.L, 1);
  o.lpn.assign(cap, 0.0);
  o.len.assign(cap, 0);
  o.tok.reset(new uint32_t[(size_t)cap * stride]);
  std::memset(&o.res, 0, sizeof(o.res));
  o.res.capacity = cap;
  o.res.stride = stride;
  o.res.logp_norm = o.lpn.data();
  o.res.lengths = o.len.data();
  o.res.tokens = o.tok.get();
  if (keys) {
    o.key.assign(cap, 0);
    o.res.key_ids = o.key.data();
  }
}

py::list key_ids(const Out &o) {
  py::list l(o.res.num_beams);
  for (uint32_t b = 0; b < o.res.num_beams; ++b) PyList_SET_ITEM(l.ptr(), b, PyLong_FromUnsignedLong(o.key[b]));
  return l;
}

py::list sentences(const Out &o) {
  py::list l(o.res.num_beams);
  for (uint32_t b = 0; b < o.res.num_beams; ++b) {
    const uint32_t n = o.len[b];
    py::list s(n);
    const uint32_t *t = o.tok.get() + (size_t)b * o.res.stride;
    for (uint32_t k = 0; k < n; ++k) PyList_SET_ITEM(s.ptr(), k, PyLong_FromUnsignedLong(t[k]));
    PyList_SET_ITEM(l.ptr(), b, s.release().ptr());
  }
  return l;
}

py::list scores(const Out &o) {
  py::list l(o.res.num_beams);
  for (uint32_t b = 0; b < o.res.num_beams; ++b) PyList_SET_ITEM(l.ptr(), b, PyFloat_FromDouble(o.lpn[b]));
  return l;
}

// A GPU search needs a workspace; the reference requires init_tbs_gpu first
// (its CPU path did not).  Without one, size a workspace to this call.
void ensure_workspace(PyTrie &t, const std::vector<Req> &reqs) {
  if (t.max_batch() > 0) return;  // an explicit workspace reports its own limits
  uint64_t K = 1, L = 1, B = 1;
  for (const Req &r : reqs) {
    K = std::max<uint64_t>(K, r.K);
    L = std::max<uint64_t>(L, r.L);
    for (uint32_t b : r.beams) B = std::max<uint64_t>(B, b);
  }
  t.init_tbs_gpu(std::max<uint64_t>(reqs.size(), 1), K, L, B, B * L, B * L, 1024);
}

ft_search_params make_params(float tt, double st, double ln, bool ee) {
  ft_search_params p;
  std::memset(&p, 0, sizeof(p));
  p.token_logp_threshold = tt;
  p.sent_logp_threshold = st;
  p.length_norm = ln;
  p.early_exit = ee ? 1 : 0;
  return p;
}

py::tuple tbs(PyTrie &trie, py::object beams, py::object topk_id, py::object topk_logp, float tt, double st,
              double ln, bool early_exit, bool /*use_gpu*/, bool return_key_ids) {
  std::vector<Req> reqs(1);
  convert_request(beams, topk_id, topk_logp, reqs[0]);
  const auto start = std::chrono::high_resolution_clock::now();
  Out o;
  prepare_out(reqs[0], o, return_key_ids);
  if (reqs[0].L == 0) throw py::value_error("tbs: beams must not be empty");
  if (reqs[0].beams[reqs[0].L - 1] != 0) {
    ensure_workspace(trie, reqs);
    ft_request fr{reqs[0].L, reqs[0].K, reqs[0].beams.data(), reqs[0].ids, reqs[0].lp};
    const ft_search_params prm = make_params(tt, st, ln, early_exit);
    py::gil_scoped_release nogil;
    check(ft_tbs_batch(trie.h(), &fr, 1, &prm, &o.res));
  }
  const auto end = std::chrono::high_resolution_clock::now();
  if (return_key_ids) return py::make_tuple(sentences(o), scores(o), msec_truncated(start, end), key_ids(o));
  return py::make_tuple(sentences(o), scores(o), msec_truncated(start, end));
}

py::tuple bs_tbs_gpu(PyTrie &trie, size_t batch_size, py::object batch_beams, py::object batch_topk_id,
                     py::object batch_topk_logp, float tt, double st, double ln, bool early_exit,
                     bool return_key_ids) {
  const size_t nb = (size_t)py::len(batch_beams), ni = (size_t)py::len(batch_topk_id),
               nl = (size_t)py::len(batch_topk_logp);
  if (nb != batch_size || ni != batch_size || nl != batch_size)
    throw py::value_error("bs_tbs_gpu: batch_size must equal the number of requests");
  std::vector<Req> reqs(batch_size);
  const bool arr3 = py::isinstance<py::array>(batch_topk_id) && py::isinstance<py::array>(batch_topk_logp);
  py::object ids_arr, lp_arr;
  if (arr3) {
    ids_arr = py::array_t<uint32_t, py::array::c_style | py::array::forcecast>::ensure(batch_topk_id);
    lp_arr = py::array_t<float, py::array::c_style | py::array::forcecast>::ensure(batch_topk_logp);
  }
  for (size_t i = 0; i < batch_size; ++i) {
    // Owning references: indexing a numpy array creates a new view object.
    py::object b = batch_beams[py::int_(i)];
    py::object ri = arr3 ? py::object(ids_arr[py::int_(i)]) : py::object(batch_topk_id[py::int_(i)]);
    py::object rl = arr3 ? py::object(lp_arr[py::int_(i)]) : py::object(batch_topk_logp[py::int_(i)]);
    convert_request(b, ri, rl, reqs[i]);
    if (reqs[i].L == 0) throw py::value_error("bs_tbs_gpu: beams must not be empty");
  }
  const auto start = std::chrono::high_resolution_clock::now();
  std::vector<Out> outs(batch_size);
  std::vector<ft_request> fr;
  std::vector<ft_result> res;
  std::vector<size_t> live;  // requests with a non-zero final beam (tbs-kernels.cu:692-697)
  for (size_t i = 0; i < batch_size; ++i) {
    prepare_out(reqs[i], outs[i], return_key_ids);
    if (reqs[i].beams[reqs[i].L - 1] == 0) continue;
    live.push_back(i);
    fr.push_back(ft_request{reqs[i].L, reqs[i].K, reqs[i].beams.data(), reqs[i].ids, reqs[i].lp});
  }
  if (!live.empty()) {
    ensure_workspace(trie, reqs);
    for (size_t i : live) res.push_back(outs[i].res);
    const ft_search_params prm = make_params(tt, st, ln, early_exit);
    {
      py::gil_scoped_release nogil;
      check(ft_tbs_batch(trie.h(), fr.data(), (uint32_t)fr.size(), &prm, res.data()));
    }
    for (size_t k = 0; k < live.size(); ++k) outs[live[k]].res = res[k];
  }
  const auto end = std::chrono::high_resolution_clock::now();
  py::list sents(batch_size), lpns(batch_size), phases(batch_size), keys(return_key_ids ? batch_size : 0);
  for (size_t i = 0; i < batch_size; ++i) {
    if (return_key_ids) PyList_SET_ITEM(keys.ptr(), i, key_ids(outs[i]).release().ptr());
    PyList_SET_ITEM(sents.ptr(), i, sentences(outs[i]).release().ptr());
    PyList_SET_ITEM(lpns.ptr(), i, scores(outs[i]).release().ptr());
    py::list ph(5);
    for (int k = 0; k < 5; ++k) PyList_SET_ITEM(ph.ptr(), k, PyFloat_FromDouble(outs[i].res.phase_ms[k]));
    PyList_SET_ITEM(phases.ptr(), i, ph.release().ptr());
  }
  if (return_key_ids) return py::make_tuple(sents, lpns, msec_truncated(start, end), phases, keys);
  return py::make_tuple(sents, lpns, msec_truncated(start, end), phases);
}

// Reader for the topk_keys.txt / topk_scores.txt proposal layout
// (tools/beam-search-helper.h:28-120): a "num_requests max_output_len topk"
// header line, then one line per (request, depth).  Rows after depth 0 are
// sorted by token id (with their scores); short rows are padded with
// UINT32_MAX / -FLT_MAX.  Ids are parsed through a float, as the reference does.
py::tuple load_topk_keys_and_scores(const std::string &dir) {
  const std::string kp = dir + "/topk_keys.txt", sp = dir + "/topk_scores.txt";
  std::cout << "Loading topk keys from " << kp << " and scores from " << sp << std::endl;
  std::ifstream kf(kp), sf(sp);
  if (!kf.is_open()) throw std::runtime_error("Error opening topk keys");
  if (!sf.is_open()) throw std::runtime_error("Error opening topk scores");
  std::string kl, sl, buf;
  std::getline(kf, kl);
  std::getline(sf, sl);
  std::stringstream kss(kl), sss(sl);
  uint32_t meta[3];
  for (int i = 0; i < 3; ++i) {
    if (!(kss >> buf)) throw std::runtime_error("malformed topk keys header");
    meta[i] = (uint32_t)std::stoi(buf);
    if (!(sss >> buf) || (uint32_t)std::stoi(buf) != meta[i])
      throw std::runtime_error("topk keys and scores headers differ");
  }
  const uint32_t num_requests = meta[0], max_len = meta[1], topk = meta[2];
  std::cout << "Parsed num_requests " << num_requests << " max_output_len " << max_len << " topk " << topk
            << std::endl;
  std::vector<std::vector<std::vector<uint32_t>>> keys(num_requests);
  std::vector<std::vector<std::vector<float>>> scores(num_requests);
  for (uint32_t r = 0; r < num_requests; ++r) {
    keys[r].resize(max_len);
    scores[r].resize(max_len);
    for (uint32_t d = 0; d < max_len; ++d) {
      auto &lk = keys[r][d];
      auto &ls = scores[r][d];
      std::getline(kf, kl);
      std::stringstream ks(kl);
      while (ks >> buf) lk.push_back((uint32_t)std::stof(buf));
      std::getline(sf, sl);
      std::stringstream ss(sl);
      while (ss >> buf) ls.push_back(std::stof(buf));
      if (lk.size() != ls.size()) throw std::runtime_error("topk keys and scores rows differ in length");
      if (d > 0) {
        std::vector<size_t> p(lk.size());
        std::iota(p.begin(), p.end(), 0);
        std::sort(p.begin(), p.end(), [&](size_t i, size_t j) { return lk[i] < lk[j]; });
        std::vector<uint32_t> k2(lk.size());
        std::vector<float> s2(ls.size());
        for (size_t i = 0; i < p.size(); ++i) {
          k2[i] = lk[p[i]];
          s2[i] = ls[p[i]];
        }
        lk.swap(k2);
        ls.swap(s2);
      }
      if (topk < lk.size()) {
        lk.resize(topk);
        ls.resize(topk);
      } else {
        while (lk.size() < topk) {
          lk.push_back(std::numeric_limits<uint32_t>::max());
          ls.push_back(-std::numeric_limits<float>::max());
        }
      }
    }
  }
  return py::make_tuple(keys, scores);
}

}  // namespace

PYBIND11_MODULE(flashtrie, m) {
  m.doc() = "B200-native trie-constrained beam search (drop-in for the FlashTrie `flashtrie` module)";
  py::class_<PyTrie>(m, "Trie")
      .def(py::init<>())
      .def("load", &PyTrie::load)
      .def("mmap", &PyTrie::mmap)
      .def("build", &PyTrie::build, py::arg("token_rows"))
      .def("total_size", [](const PyTrie &t) { return t.info().total_size; })
      .def("io_size", [](const PyTrie &t) { return t.info().io_size; })
      .def("num_tries", [](const PyTrie &t) { return t.info().num_tries; })
      .def("num_keys", [](const PyTrie &t) { return t.info().num_keys; })
      .def("num_nodes", [](const PyTrie &t) { return t.info().num_nodes; })
      .def("save", &PyTrie::save)
      .def("clear", &PyTrie::clear)
      .def("init_tbs_gpu", &PyTrie::init_tbs_gpu, py::arg("max_batch_size"), py::arg("max_num_topk") = 1024,
           py::arg("max_num_outpos") = 64, py::arg("max_num_out_beams") = 8192,
           py::arg("max_num_out_tokens") = 8192 * 64, py::arg("max_num_inter_beams") = 1024 * 1024,
           py::arg("radix_topk_threshold") = 1024)
      .def("get_max_batch_size", &PyTrie::max_batch)
      // Extensions beyond the reference surface:
      //   build_flat(tokens u32[total], offsets u64[n+1]) builds from flat arrays;
      //   ft_handle() is the ft_trie* of the C ABI (include/flashtrie_b200.h),
      //   for callers that drive ft_tbs_batch_device on their own streams.
      .def("build_flat", [](PyTrie &t, py::array_t<uint32_t, py::array::c_style | py::array::forcecast> tokens,
                            py::array_t<uint64_t, py::array::c_style | py::array::forcecast> offsets) {
        if (tokens.ndim() != 1 || offsets.ndim() != 1 || offsets.size() < 1)
          throw py::value_error("build_flat: tokens and offsets must be 1-D, offsets non-empty");
        const uint64_t n = (uint64_t)offsets.size() - 1;
        if (offsets.data()[n] > (uint64_t)tokens.size()) throw py::value_error("build_flat: offsets exceed tokens");
        const uint32_t *tp = tokens.data();
        const uint64_t *op = offsets.data();
        py::gil_scoped_release nogil;
        check(ft_trie_build(t.h(), tp, op, n));
      }, py::arg("tokens"), py::arg("offsets"))
      .def("ft_handle", [](const PyTrie &t) { return (uintptr_t)t.h(); });

  m.def("tbs", &tbs, py::arg("trie"), py::arg("beams"), py::arg("topk_id"), py::arg("topk_logp"),
        py::arg("token_logp_threshold"), py::arg("sents_logp_threshold"), py::arg("length_norm"),
        py::arg("early_exit"), py::arg("use_gpu") = false, py::kw_only(), py::arg("return_key_ids") = false);
  m.def("bs_tbs_gpu", &bs_tbs_gpu, py::arg("trie"), py::arg("batch_size"), py::arg("batch_beams"),
        py::arg("batch_topk_id"), py::arg("batch_topk_logp"), py::arg("token_logp_threshold"),
        py::arg("sents_logp_threshold"), py::arg("length_norm"), py::arg("early_exit"), py::kw_only(),
        py::arg("return_key_ids") = false);
  m.def("load_topk_keys_and_scores", &load_topk_keys_and_scores, py::arg("dataset_dir"));
}
