// Stand-in for a LAMMPS pair style written against DeePMD's header-only C++
// API: it includes the b200dp shim as deepmd::hpp (the way the reference's
// pair style selects deepmd_compat, components/lammps-deepmd-plugin/src/
// pair_base.h:9-24), builds an InputNlist from a LAMMPS-style full list with
// ghost atoms and special-bond mask bits, calls DeepPot::compute as
// PairDeepMD::compute does (pair_deepmd.cpp:356-390), folds the ghost forces
// back onto their owners (LAMMPS reverse communication) and writes the result.
//
//   pair_stub <model> <input.bin> <output.bin>
// input:  int32 nlocal, nghost, nflat; fp64 coord[nall*3]; int32 atype[nall];
//         int32 owner[nghost]; int32 numneigh[nlocal]; int32 flat[nflat]
// output: fp64 energy, force[nlocal*3], virial[9], energy_from_atomic,
//         atom_energy[nlocal], virial_from_atomic[9]
#define B200DP_AS_DEEPMD_HPP
#include "b200dp_deepmd.hpp"

#include <cstdio>
#include <string>
#include <vector>

namespace deepmd_compat = deepmd::hpp;

constexpr int kNeighMask = 0x1FFFFFFF;  // LAMMPS NEIGHMASK: the top bits carry special-bond flags

template <class T>
static bool rd(FILE* f, T* p, size_t n) {
  return fread(p, sizeof(T), n, f) == n;
}

int main(int argc, char** argv) {
  if (argc != 4 && argc != 5) return 2;  // model, input, output[, "fp64"]
  FILE* in = fopen(argv[2], "rb");
  if (!in) return 3;
  int hdr[3];
  if (!rd(in, hdr, 3)) return 4;
  const int nlocal = hdr[0], nghost = hdr[1], nflat = hdr[2], nall = nlocal + nghost;
  std::vector<double> coord(3 * (size_t)nall);
  std::vector<int> atype(nall), owner(nghost), numneigh(nlocal), flat(nflat), ilist(nlocal);
  if (!rd(in, coord.data(), coord.size()) || !rd(in, atype.data(), atype.size()) ||
      !rd(in, owner.data(), owner.size()) || !rd(in, numneigh.data(), numneigh.size()) ||
      !rd(in, flat.data(), flat.size()))
    return 5;
  fclose(in);
  std::vector<int*> firstneigh(nlocal);
  size_t off = 0;
  for (int i = 0; i < nlocal; ++i) {
    ilist[i] = i;
    firstneigh[i] = flat.data() + off;
    off += numneigh[i];
  }
  try {
    deepmd_compat::DeepPot deep_pot;
    if (argc > 4 && std::string(argv[4]) == "fp64") deep_pot.set_precision(B200DP_FP64);
    deep_pot.init(argv[1], 0, "");
    std::string tm;
    deep_pot.get_type_map(tm);
    if (deep_pot.numb_types() < 1 || deep_pot.cutoff() <= 0 || deep_pot.dim_fparam() != 0) return 6;
    deepmd_compat::InputNlist lmp_list(nlocal, ilist.data(), numneigh.data(), firstneigh.data(), 0, nullptr,
                                       nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 1);
    lmp_list.set_mask(kNeighMask);
    std::vector<double> dbox;  // ghosts given: no box
    double dener = 0;
    std::vector<double> dforce, dvirial;
    int ago = 0;
    deep_pot.compute(dener, dforce, dvirial, coord, atype, dbox, nghost, lmp_list, ago);
    double dener2 = 0;
    std::vector<double> dforce2, dvirial2, deatom, dvatom;
    ago = 1;
    deep_pot.compute(dener2, dforce2, dvirial2, deatom, dvatom, coord, atype, dbox, nghost, lmp_list, ago);
    // reverse communication: ghost forces onto their owners
    for (int g = 0; g < nghost; ++g)
      for (int c = 0; c < 3; ++c) dforce[3 * owner[g] + c] += dforce[3 * (nlocal + g) + c];
    double esum = 0, vsum[9] = {0};
    for (int i = 0; i < nlocal; ++i) esum += deatom[i];
    for (int i = 0; i < nall; ++i)
      for (int k = 0; k < 9; ++k) vsum[k] += dvatom[9 * i + k];
    FILE* out = fopen(argv[3], "wb");
    if (!out) return 7;
    fwrite(&dener, sizeof(double), 1, out);
    fwrite(dforce.data(), sizeof(double), 3 * (size_t)nlocal, out);
    fwrite(dvirial.data(), sizeof(double), 9, out);
    fwrite(&esum, sizeof(double), 1, out);
    fwrite(deatom.data(), sizeof(double), nlocal, out);
    fwrite(vsum, sizeof(double), 9, out);
    fclose(out);
  } catch (deepmd_compat::deepmd_exception& e) {
    fprintf(stderr, "%s\n", e.what());
    return 8;
  }
  return 0;
}
