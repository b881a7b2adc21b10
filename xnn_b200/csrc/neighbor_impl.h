// Cell-list neighbour search shared by the CUDA kernel and the C++/OpenMP CPU twin.
//
// Atoms are binned into n0 x n1 x n2 cells of the (triclinic) cell in fractional
// coordinates, each at least one cutoff wide along its plane normal, or a single cell
// with k image layers when the box is thinner than the cutoff. Receiver i visits the
// cells c_i + (-k..k)^3; for a periodic axis the visited cell wraps and carries an
// integer image shift, for an open axis cells outside the box are skipped. Every pair
// (j, image s) is visited at most once per receiver. Two passes over the same loop
// (count, then write at the receiver's prefix-sum offset) give edges grouped by
// receiver in a fixed order without atomics.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define XNN_NB_HD __host__ __device__ __forceinline__
#else
#define XNN_NB_HD inline
#endif

struct NbParams {
  const double* pos;          // (N, 3), wrapped along periodic axes
  double cell[9];             // rows are lattice vectors
  int64_t ncell[3];
  int64_t k[3];
  int pbc[3];
  const int64_t* atom_cell;   // (N,) linear cell index of every atom
  const int64_t* sorted;      // (N,) atoms ordered by cell
  const int64_t* cell_start;  // (ncells + 1,)
  double cutoff2;
  int self_interaction;
  int64_t N;
  int64_t r0;                 // receivers r0 .. r0 + M - 1 are searched (all atoms are candidates)
  int64_t M;
};

// Visits every candidate pair of receiver i; fn(j, s0, s1, s2) for pairs inside the cutoff.
template <typename F>
XNN_NB_HD void nb_visit(const NbParams& p, int64_t i, F&& fn) {
  const int64_t ci = p.atom_cell[i];
  const int64_t c2 = ci % p.ncell[2];
  const int64_t c1 = (ci / p.ncell[2]) % p.ncell[1];
  const int64_t c0 = ci / (p.ncell[2] * p.ncell[1]);
  const double xi = p.pos[3 * i], yi = p.pos[3 * i + 1], zi = p.pos[3 * i + 2];
  for (int64_t d0 = -p.k[0]; d0 <= p.k[0]; ++d0) {
    int64_t a0 = c0 + d0, s0 = 0;
    if (p.pbc[0]) {
      s0 = (a0 >= 0) ? a0 / p.ncell[0] : -((-a0 + p.ncell[0] - 1) / p.ncell[0]);
      a0 -= s0 * p.ncell[0];
    } else if (a0 < 0 || a0 >= p.ncell[0]) {
      continue;
    }
    for (int64_t d1 = -p.k[1]; d1 <= p.k[1]; ++d1) {
      int64_t a1 = c1 + d1, s1 = 0;
      if (p.pbc[1]) {
        s1 = (a1 >= 0) ? a1 / p.ncell[1] : -((-a1 + p.ncell[1] - 1) / p.ncell[1]);
        a1 -= s1 * p.ncell[1];
      } else if (a1 < 0 || a1 >= p.ncell[1]) {
        continue;
      }
      for (int64_t d2 = -p.k[2]; d2 <= p.k[2]; ++d2) {
        int64_t a2 = c2 + d2, s2 = 0;
        if (p.pbc[2]) {
          s2 = (a2 >= 0) ? a2 / p.ncell[2] : -((-a2 + p.ncell[2] - 1) / p.ncell[2]);
          a2 -= s2 * p.ncell[2];
        } else if (a2 < 0 || a2 >= p.ncell[2]) {
          continue;
        }
        const double sx = s0 * p.cell[0] + s1 * p.cell[3] + s2 * p.cell[6];
        const double sy = s0 * p.cell[1] + s1 * p.cell[4] + s2 * p.cell[7];
        const double sz = s0 * p.cell[2] + s1 * p.cell[5] + s2 * p.cell[8];
        const bool zero_shift = (s0 == 0 && s1 == 0 && s2 == 0);
        const int64_t cell = (a0 * p.ncell[1] + a1) * p.ncell[2] + a2;
        for (int64_t q = p.cell_start[cell]; q < p.cell_start[cell + 1]; ++q) {
          const int64_t j = p.sorted[q];
          if (j == i && zero_shift && !p.self_interaction) continue;
          const double dx = p.pos[3 * j] + sx - xi;
          const double dy = p.pos[3 * j + 1] + sy - yi;
          const double dz = p.pos[3 * j + 2] + sz - zi;
          if (dx * dx + dy * dy + dz * dz < p.cutoff2) fn(j, s0, s1, s2);
        }
      }
    }
  }
}
