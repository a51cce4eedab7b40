// Invariants of the tensor-core forward's work split (TileSplit / plan_split in
// murmurative_attention_b200/csrc/murm_common.cuh), checked by brute force over many shapes:
// every (b,h) x tile unit belongs to exactly one CTA, CTA runs are non-empty and at most
// kMaxSplitCtas, cta_of() finds the owner, a pair's partial indices (CTA - first CTA of the pair)
// are 0..parts-1 in token order, and max_parts() bounds parts() (the workspace is sized by it).
// Prints "ok <shapes>" or the first failure; exit status 0 on success.
#include <cstdio>
#include <vector>

#include "../murmurative_attention_b200/csrc/murm_common.cuh"

using namespace murm;

int main() {
  const int BHs[] = {1, 2, 3, 5, 7, 8, 15, 16, 17, 32, 33, 64, 100, 147, 148, 149, 150, 160, 200, 300, 1000, 5000};
  const int Ns[] = {1, 2, 63, 64, 127, 128, 129, 255, 256, 300, 520, 1000, 1024, 4096, 8192, 16384};
  const int tiles[] = {kTile, kBwdTile};
  int shapes = 0;
  for (int tile : tiles)
    for (int BH : BHs)
      for (int N : Ns) {
        TileSplit s;
        plan_split(BH, N, tile, kMaxSplitCtas, &s);
        const int tpb = (N + tile - 1) / tile, U = BH * tpb;
        ++shapes;
        if (s.G < 1 || s.G > kMaxSplitCtas || s.tpb != tpb || s.start[0] != 0 || s.start[s.G] != U) {
          printf("bad plan BH=%d N=%d tile=%d\n", BH, N, tile);
          return 1;
        }
        std::vector<int> owner(U, -1);
        for (int c = 0; c < s.G; ++c) {
          if (s.start[c + 1] <= s.start[c]) {
            printf("empty run BH=%d N=%d tile=%d c=%d\n", BH, N, tile, c);
            return 1;
          }
          for (int u = s.start[c]; u < s.start[c + 1]; ++u) owner[u] = c;
        }
        for (int u = 0; u < U; ++u)
          if (owner[u] < 0 || s.cta_of(u) != owner[u]) {
            printf("cta_of BH=%d N=%d tile=%d u=%d\n", BH, N, tile, u);
            return 1;
          }
        const int bound = max_parts(s);
        for (int bh = 0; bh < BH; ++bh) {
          const int p = s.parts(bh);
          if (p > bound) {
            printf("parts %d > bound %d BH=%d N=%d tile=%d\n", p, bound, BH, N, tile);
            return 1;
          }
          int last = -1;
          for (int t = 0; t < tpb; ++t) {
            const int pi = owner[bh * tpb + t] - s.first_cta(bh);
            if (pi < 0 || pi >= p || pi < last) {
              printf("partial index BH=%d N=%d tile=%d bh=%d t=%d\n", BH, N, tile, bh, t);
              return 1;
            }
            last = pi;
          }
        }
      }
  printf("ok %d\n", shapes);
  return 0;
}
