/*
 * b200dp_deepmd.hpp — DeePMD-kit C++ API shim over the b200dp C ABI.
 *
 * Header-only.  Gives a LAMMPS pair style written against DeePMD's
 * header-only C++ wrapper (`deepmd::hpp`, included by the reference's pair
 * style as deepmd.hpp: components/lammps-deepmd-plugin/src/pair_base.h:9-24)
 * the subset of that API the pair style calls
 * (components/lammps-deepmd-plugin/src/pair_deepmd.cpp:356-390, 594, 668-697,
 * 1000): DeepPot::init / cutoff / numb_types / dim_fparam / dim_aparam /
 * get_type_map and the compute overloads with and without a LAMMPS neighbour
 * list, InputNlist with its neighbour mask, and deepmd_exception.
 *
 * By default the classes live in namespace b200dp_deepmd.  Defining
 * B200DP_AS_DEEPMD_HPP before including this header also exposes them as
 * deepmd::hpp, so a pair style that says `namespace deepmd_compat =
 * deepmd::hpp;` compiles against this header in place of deepmd.hpp.
 *
 * Precision: a DeepPot is constructed for the mixed-precision engine
 * (DeepPot(), DeePMD's default constructor) or for a given one
 * (DeepPot(B200DP_FP64)); set_precision() changes it before init.  No
 * environment variable is read.  The GPU is gpu_rank % (number of visible
 * devices).
 *
 * Conventions are DeePMD's: coord [nall*3], atype [nall] (0-based), box [9]
 * (empty: no periodic box), nghost trailing ghost atoms; force [nall*3]
 * (ghost rows are partial forces for the caller's reverse communication),
 * virial [9], atom_energy [nall] (ghost rows zero), atom_virial [nall*9].
 */
#ifndef B200DP_DEEPMD_HPP
#define B200DP_DEEPMD_HPP

#include <cuda_runtime_api.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "b200dp.h"

namespace b200dp_deepmd {

struct deepmd_exception : public std::runtime_error {
  explicit deepmd_exception(const std::string& msg) : std::runtime_error("b200dp: " + msg) {}
};

// LAMMPS neighbour list view (inum, ilist, numneigh, firstneigh).  The
// communication fields of DeePMD's InputNlist are accepted and kept, but this
// engine needs only the list itself: ghosts arrive as coordinates.
struct InputNlist {
  int inum = 0;
  int* ilist = nullptr;
  int* numneigh = nullptr;
  int** firstneigh = nullptr;
  int nswap = 0;
  int* sendnum = nullptr;
  int* recvnum = nullptr;
  int* firstrecv = nullptr;
  int** sendlist = nullptr;
  int* sendproc = nullptr;
  int* recvproc = nullptr;
  void* world = nullptr;
  int nprocs = 1;
  int mask = -1;
  int* mapping = nullptr;
  InputNlist() = default;
  InputNlist(int inum_, int* ilist_, int* numneigh_, int** firstneigh_)
      : inum(inum_), ilist(ilist_), numneigh(numneigh_), firstneigh(firstneigh_) {}
  InputNlist(int inum_, int* ilist_, int* numneigh_, int** firstneigh_, int nswap_, int* sendnum_, int* recvnum_,
             int* firstrecv_, int** sendlist_, int* sendproc_, int* recvproc_, void* world_, int nprocs_ = 1)
      : inum(inum_), ilist(ilist_), numneigh(numneigh_), firstneigh(firstneigh_), nswap(nswap_),
        sendnum(sendnum_), recvnum(recvnum_), firstrecv(firstrecv_), sendlist(sendlist_), sendproc(sendproc_),
        recvproc(recvproc_), world(world_), nprocs(nprocs_) {}
  void set_mask(int m) { mask = m; }
  void set_mapping(int* m) { mapping = m; }
};

class DeepBaseModel {
 public:
  virtual ~DeepBaseModel() = default;
  virtual double cutoff() const = 0;
  virtual int numb_types() const = 0;
  virtual int numb_types_spin() const { return 0; }
  virtual int dim_fparam() const { return 0; }
  virtual int dim_aparam() const { return 0; }
  virtual int dim_chg_spin() const { return 0; }
  virtual void get_type_map(std::string& type_map) = 0;
};

class DeepPot : public DeepBaseModel {
 public:
  DeepPot() = default;
  explicit DeepPot(int precision) : precision_(precision) {}
  // B200DP_FP64 or B200DP_MIXED, before init
  void set_precision(int precision) {
    if (eng_) throw deepmd_exception("set_precision must come before init");
    precision_ = precision;
  }
  explicit DeepPot(const std::string& model, const int& gpu_rank = 0, const std::string& file_content = "") {
    init(model, gpu_rank, file_content);
  }
  ~DeepPot() override {
    if (eng_) b200dp_destroy(eng_);
  }
  DeepPot(const DeepPot&) = delete;
  DeepPot& operator=(const DeepPot&) = delete;

  // file_content (DeePMD's in-memory model bytes) is not supported: the model
  // is read from `model`.
  void init(const std::string& model, const int& gpu_rank = 0, const std::string& file_content = "") {
    if (eng_) throw deepmd_exception("already initialised");
    if (!file_content.empty()) throw deepmd_exception("in-memory model content is not supported; pass a file");
    b200dp_options opt;
    b200dp_options_default(&opt);
    opt.precision = precision_;
    int ndev = 1;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev < 1) ndev = 1;
    opt.device = gpu_rank >= 0 ? gpu_rank % ndev : 0;
    if (b200dp_create(model.c_str(), &opt, &eng_) != B200DP_OK) {
      eng_ = nullptr;
      throw deepmd_exception("cannot load model " + model);
    }
    b200dp_model_info_get(eng_, &info_);
  }

  double cutoff() const override { return info_.rcut; }
  int numb_types() const override { return info_.ntypes; }
  void get_type_map(std::string& type_map) override {
    type_map.clear();
    for (int t = 0; t < info_.ntypes; ++t) type_map += (t ? " type" : "type") + std::to_string(t);
  }
  template <typename T>
  void set_charge_spin(const std::vector<T>&) {}

  // Periodic box (or none), no neighbour list.
  template <typename E, typename V>
  void compute(E& ener, std::vector<V>& force, std::vector<V>& virial, const std::vector<V>& coord,
               const std::vector<int>& atype, const std::vector<V>& box, const std::vector<V>& fparam = {},
               const std::vector<V>& aparam = {}) {
    run<E, V>(ener, force, virial, nullptr, nullptr, coord, atype, box, 0, nullptr, fparam, aparam);
  }
  template <typename E, typename V>
  void compute(E& ener, std::vector<V>& force, std::vector<V>& virial, std::vector<V>& atom_energy,
               std::vector<V>& atom_virial, const std::vector<V>& coord, const std::vector<int>& atype,
               const std::vector<V>& box, const std::vector<V>& fparam = {}, const std::vector<V>& aparam = {}) {
    run(ener, force, virial, &atom_energy, &atom_virial, coord, atype, box, 0, nullptr, fparam, aparam);
  }
  // LAMMPS path: nghost trailing ghosts and the pair style's neighbour list.
  template <typename E, typename V>
  void compute(E& ener, std::vector<V>& force, std::vector<V>& virial, const std::vector<V>& coord,
               const std::vector<int>& atype, const std::vector<V>& box, const int nghost, const InputNlist& lmp_list,
               const int& ago, const std::vector<V>& fparam = {}, const std::vector<V>& aparam = {},
               const std::vector<V>& charge_spin = {}) {
    (void)ago;
    (void)charge_spin;
    run<E, V>(ener, force, virial, nullptr, nullptr, coord, atype, box, nghost, &lmp_list, fparam, aparam);
  }
  template <typename E, typename V>
  void compute(E& ener, std::vector<V>& force, std::vector<V>& virial, std::vector<V>& atom_energy,
               std::vector<V>& atom_virial, const std::vector<V>& coord, const std::vector<int>& atype,
               const std::vector<V>& box, const int nghost, const InputNlist& lmp_list, const int& ago,
               const std::vector<V>& fparam = {}, const std::vector<V>& aparam = {},
               const std::vector<V>& charge_spin = {}) {
    (void)ago;
    (void)charge_spin;
    run(ener, force, virial, &atom_energy, &atom_virial, coord, atype, box, nghost, &lmp_list, fparam, aparam);
  }

  b200dp_engine* engine() const { return eng_; }

 private:
  template <typename E, typename V>
  void run(E& ener, std::vector<V>& force, std::vector<V>& virial, std::vector<V>* atom_energy,
           std::vector<V>* atom_virial, const std::vector<V>& coord, const std::vector<int>& atype,
           const std::vector<V>& box, int nghost, const InputNlist* nl, const std::vector<V>& fparam,
           const std::vector<V>& aparam) {
    if (!eng_) throw deepmd_exception("not initialised");
    if (!fparam.empty() || !aparam.empty()) throw deepmd_exception("frame / atomic parameters are not supported");
    const int nall = (int)atype.size();
    const int nloc = nall - nghost;
    if (coord.size() != 3 * (size_t)nall || nloc < 0) throw deepmd_exception("coord / atype / nghost sizes differ");
    std::vector<double> x(coord.begin(), coord.end()), b(box.begin(), box.end()), f(3 * (size_t)nall), w(9);
    std::vector<double> ae, av;
    if (atom_energy) ae.assign(std::max(nloc, 0), 0.0);
    if (atom_virial) av.assign(9 * (size_t)nall, 0.0);
    double e = 0.0;
    b200dp_status st;
    if (nl) {
      // apply the LAMMPS neighbour mask to a private copy of the list
      std::vector<int> flat, cnt(nl->inum), il(nl->ilist, nl->ilist + nl->inum);
      for (int r = 0; r < nl->inum; ++r) {
        cnt[r] = nl->numneigh[r];
        for (int k = 0; k < cnt[r]; ++k) flat.push_back(nl->firstneigh[r][k] & nl->mask);
      }
      std::vector<int*> first(nl->inum);
      size_t off = 0;
      for (int r = 0; r < nl->inum; ++r) {
        first[r] = flat.data() + off;
        off += cnt[r];
      }
      b200dp_nlist list{nl->inum, il.data(), cnt.data(), first.data()};
      st = b200dp_compute_host_nlist(eng_, nloc, nghost, x.data(), atype.data(), &list, &e, f.data(), w.data(),
                                     atom_energy ? ae.data() : nullptr, atom_virial ? av.data() : nullptr);
    } else {
      st = b200dp_compute_host(eng_, nloc, nghost, x.data(), atype.data(), b.empty() ? nullptr : b.data(), &e,
                               f.data(), w.data(), atom_energy ? ae.data() : nullptr,
                               atom_virial ? av.data() : nullptr);
    }
    if (st != B200DP_OK) throw deepmd_exception(b200dp_last_error(eng_));
    ener = (E)e;
    force.assign(f.begin(), f.end());
    virial.assign(w.begin(), w.end());
    if (atom_energy) {
      atom_energy->assign((size_t)nall, (V)0);
      for (int i = 0; i < nloc; ++i) (*atom_energy)[i] = (V)ae[i];
    }
    if (atom_virial) atom_virial->assign(av.begin(), av.end());
  }

  b200dp_engine* eng_ = nullptr;
  int precision_ = B200DP_MIXED;
  b200dp_model_info info_{};
};

}  // namespace b200dp_deepmd

#ifdef B200DP_AS_DEEPMD_HPP
namespace deepmd {
namespace hpp {
using b200dp_deepmd::deepmd_exception;
using b200dp_deepmd::DeepBaseModel;
using b200dp_deepmd::DeepPot;
using b200dp_deepmd::InputNlist;
}  // namespace hpp
}  // namespace deepmd
#endif

#endif  // B200DP_DEEPMD_HPP
