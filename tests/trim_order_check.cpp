// Check (test infrastructure, CPU): the partition formulation that the device cloud trim uses
// reproduces the permutation std::nth_element leaves behind.
//
// ObjCloud::add (scenemap src/cloud.cpp:114-123) trims a cloud with
//   std::nth_element(pts.begin(), pts.begin() + (n - keep), pts.end(), by seq)
// and keeps the last `keep` elements in the order nth_element left them; later code samples the
// cloud with a stride, so that order is an output.  The device reproduces libstdc++'s selection
// (median-of-three pivot, unguarded Hoare partition, depth limit 2*floor(log2 n), insertion
// sort below 4 elements) with each partition computed in parallel: with L = the positions
// holding a key >= pivot (ascending) and R = the positions holding a key <= pivot (descending),
// the sequential partition swaps L[i] <-> R[i] for every i with L[i] < R[i], and returns
// L[0] when no swap happened, else min(L[k], R[k-1]) for the k swaps made.
//
// Build: g++ -O2 -std=c++17 trim_order_check.cpp; run: ./a.out [trials]; prints "ok N" or the
// first mismatch and exits 1.
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <random>
#include <vector>

struct El {
  uint32_t seq, idx;
};

// one partition of [first, last) around the key at `first`, the pairing rule above
static long partition_pairs(std::vector<El>& a, long first, long last) {
  const uint32_t p = a[first].seq;
  std::vector<long> L, R;
  for (long j = first + 1; j < last; ++j)
    if (!(a[j].seq < p)) L.push_back(j);
  for (long j = last - 1; j > first; --j)
    if (!(p < a[j].seq)) R.push_back(j);
  long k = 0;
  const long nk = (long)std::min(L.size(), R.size());
  while (k < nk && L[k] < R[k]) ++k;
  for (long i = 0; i < k; ++i) std::swap(a[L[i]], a[R[i]]);
  if (k == 0) return L[0];
  const long lk = k < (long)L.size() ? L[k] : last;
  return std::min(lk, R[k - 1]);
}

static void median_to_first(std::vector<El>& a, long r, long x, long y, long z) {
  auto lt = [&](long i, long j) { return a[i].seq < a[j].seq; };
  long m;
  if (lt(x, y)) m = lt(y, z) ? y : (lt(x, z) ? z : x);
  else m = lt(x, z) ? x : (lt(y, z) ? z : y);
  std::swap(a[r], a[m]);
}

// returns false when the depth limit runs out (the device then reports an error)
static bool select_order(std::vector<El>& a, long nth) {
  long first = 0, last = (long)a.size();
  if (first == last || nth == last) return true;
  long lg = 0;
  for (long n = last - first; n > 1; n >>= 1) ++lg;
  long depth = 2 * lg;
  while (last - first > 3) {
    if (depth == 0) return false;
    --depth;
    const long mid = first + (last - first) / 2;
    median_to_first(a, first, first + 1, mid, last - 1);
    const long cut = partition_pairs(a, first, last);
    if (cut <= nth) first = cut;
    else last = cut;
  }
  // stable insertion sort of the last few elements
  for (long i = first + 1; i < last; ++i) {
    const El v = a[i];
    long j = i;
    while (j > first && v.seq < a[j - 1].seq) { a[j] = a[j - 1]; --j; }
    a[j] = v;
  }
  return true;
}

int main(int argc, char** argv) {
  const int trials = argc > 1 ? atoi(argv[1]) : 2000;
  std::mt19937_64 rng(12345);
  int depth_out = 0;
  for (int t = 0; t < trials; ++t) {
    // clouds: runs of equal seq (one per add call), newest last, with overwritten voxels
    // scattered back to older positions; sizes across the cap, a few tiny ones
    const long n = t < 50 ? 1 + (long)(rng() % 12) : 7000 + (long)(rng() % 9000);
    const int calls = 1 + (int)(rng() % 60);
    std::vector<El> a((size_t)n);
    for (long i = 0; i < n; ++i) a[(size_t)i] = El{(uint32_t)(1 + (i * calls) / n), (uint32_t)i};
    for (long i = 0; i < n / 7; ++i) a[(size_t)(rng() % n)].seq = (uint32_t)(1 + rng() % (calls + 1));
    if (t % 5 == 0) for (auto& e : a) e.seq = (uint32_t)(1 + rng() % 3);   // very few distinct keys
    const long keep = std::max<long>(1, std::min<long>(n, 7200));
    const long nth = n - keep;
    std::vector<El> ref = a, mine = a;
    std::nth_element(ref.begin(), ref.begin() + nth, ref.end(), [](const El& x, const El& y) { return x.seq < y.seq; });
    if (!select_order(mine, nth)) { ++depth_out; continue; }
    for (long i = 0; i < n; ++i)
      if (ref[(size_t)i].idx != mine[(size_t)i].idx) {
        printf("mismatch trial %d n %ld at %ld: ref %u mine %u\n", t, n, i, ref[(size_t)i].idx, mine[(size_t)i].idx);
        return 1;
      }
  }
  printf("ok %d depth_limit_hit %d\n", trials, depth_out);
  return 0;
}
