// Host-side batch encoder: positions -> the collated MantisNet batch arrays.
//
// The C++ counterpart of the package's numpy builder (builder.py: build +
// collate + relay views), itself checked bit-exact against the reference
// builder's fixtures (reference python/mantisnet/mantisnet/builder.py:486-956,
// relay.py:48-94; the production Rust builder is
// crates/models/mantisnet/src/encoder.rs). Every array, order included, is
// part of the representation contract, so each step below states the
// ordering rule it follows:
//
//   windows       ascending key pack(start) * 4 + axis over every (axis,
//                 start) whose six cells hold a stone;
//   incidence     window-major, slot-minor;
//   radius edges  destination cell-major, source stone-minor (cells within
//                 hex distance 8 of a stone);
//   adjacency     (destination, source, axis) ascending over distance-one
//                 pairs of legal cells;
//   decoder rows  legal-cell-major, then axis, then offset k of the window
//                 start before the cell (only live windows); action rows ride
//                 the same order;
//   relay views   stable sorts of the decoder rows by cell, window, class.
//
// Work: phase 1 builds each position's graph on its own (a thread per slice
// of positions); phase 2 writes the batch into caller-owned buffers, each
// position's rows at its offsets, then the batch-wide relay sorts (counting
// sorts, stable). Coordinate lookups go through open-addressing hash tables
// keyed by the packed coordinate, so a position costs O(cells) whatever its
// extent.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace mb {
namespace enc {

constexpr int W = 6;              // window length
constexpr int GLOBAL_ROWS = 4;
constexpr int LEGAL_RADIUS = 8;
constexpr int64_t NEAREST_UNREACHED = 9;
constexpr int TACTICAL = 11;
constexpr int THREAT_CAP = 8;
constexpr int ORBIT_SPAN = 12;
constexpr int NPAT = 729;         // 3^6 raw window patterns
constexpr int DEC_CLASSES = 726;
constexpr int EMPTY_ORBITS = 3;
constexpr int ACT_OWN = 0, ACT_OPP = 1, ACT_EMPTY = 2, ACT_MIXED = 3;
constexpr int64_t QSHIFT = int64_t(1) << 21;
constexpr int AX[3][2] = {{1, 0}, {0, 1}, {1, -1}};  // line axes Q, R, QR

inline int64_t pack(int64_t q, int64_t r) { return q * QSHIFT + r; }

// ---------------------------------------------------------------- tables --
// The closed vocabularies, derived as the package's vocab.py derives them
// (orbits ranked by their smallest member); a test compares every entry.
struct Tables {
  int pow3[W];
  int rank[NPAT];           // window pattern -> reversal class (-1 for empty)
  int occ[NPAT][W];         // (pattern, occupied slot) class
  int dec[NPAT][W];         // (pattern, empty slot) class, nonempty patterns
  int post1[NPAT][W];       // (pattern, own-stone slot) class
  int orbit48[2 * ORBIT_SPAN + 1][2 * ORBIT_SPAN + 1];
  int slot_orbit[W];
  // radius-8 disk without its centre, in (dq, dr) row-major order
  std::vector<int> disk_q, disk_r, disk_dist, disk_orbit, disk_on_axis;

  Tables() {
    for (int k = 0, p = 1; k < W; ++k, p *= 3) pow3[k] = p;
    int digit[NPAT][W], rev[NPAT];
    for (int p = 0; p < NPAT; ++p) {
      rev[p] = 0;
      for (int k = 0; k < W; ++k) digit[p][k] = (p / pow3[k]) % 3;
      for (int k = 0; k < W; ++k) rev[p] += digit[p][W - 1 - k] * pow3[k];
    }
    std::vector<int> reps;
    for (int p = 1; p < NPAT; ++p) reps.push_back(std::min(p, rev[p]));
    std::sort(reps.begin(), reps.end());
    reps.erase(std::unique(reps.begin(), reps.end()), reps.end());
    rank[0] = -1;
    for (int p = 1; p < NPAT; ++p)
      rank[p] = (int)(std::lower_bound(reps.begin(), reps.end(), std::min(p, rev[p])) - reps.begin());
    auto orbit_rank = [&](int (*table)[W], auto in_mask) {
      std::vector<int> r;
      for (int p = 0; p < NPAT; ++p)
        for (int s = 0; s < W; ++s)
          if (in_mask(p, s)) r.push_back(std::min(p * W + s, rev[p] * W + (W - 1 - s)));
      std::sort(r.begin(), r.end());
      r.erase(std::unique(r.begin(), r.end()), r.end());
      for (int p = 0; p < NPAT; ++p)
        for (int s = 0; s < W; ++s)
          table[p][s] = in_mask(p, s) ? (int)(std::lower_bound(r.begin(), r.end(),
                                                               std::min(p * W + s, rev[p] * W + (W - 1 - s))) -
                                              r.begin())
                                      : -1;
    };
    orbit_rank(dec, [&](int p, int s) { return digit[p][s] == 0 && p != 0; });
    orbit_rank(occ, [&](int p, int s) { return digit[p][s] != 0; });
    orbit_rank(post1, [&](int p, int s) { return digit[p][s] == 1; });
    for (int k = 0; k < W; ++k) slot_orbit[k] = std::min(k, W - 1 - k);

    // D6 displacement orbits within distance 12, ordered by (distance,
    // smallest image); images are the six rotations of (q, r) and of (r, q).
    struct Rep { int d, a, b; bool operator<(const Rep& o) const { return d != o.d ? d < o.d : (a != o.a ? a < o.a : b < o.b); }
                 bool operator==(const Rep& o) const { return d == o.d && a == o.a && b == o.b; } };
    auto rep_of = [](int q, int r) {
      const int d = std::max(std::abs(q), std::max(std::abs(r), std::abs(q + r)));
      Rep best{d, 1 << 30, 1 << 30};
      const int seeds[2][2] = {{q, r}, {r, q}};
      for (auto& sd : seeds) {
        int a = sd[0], b = sd[1];
        for (int i = 0; i < 6; ++i) {
          if (a < best.a || (a == best.a && b < best.b)) { best.a = a; best.b = b; }
          const int na = -b, nb = a + b;
          a = na; b = nb;
        }
      }
      return best;
    };
    std::vector<Rep> all;
    for (int q = -ORBIT_SPAN; q <= ORBIT_SPAN; ++q)
      for (int r = -ORBIT_SPAN; r <= ORBIT_SPAN; ++r) {
        const int d = std::max(std::abs(q), std::max(std::abs(r), std::abs(q + r)));
        if (d >= 1 && d <= ORBIT_SPAN) all.push_back(rep_of(q, r));
      }
    std::sort(all.begin(), all.end());
    all.erase(std::unique(all.begin(), all.end()), all.end());
    for (int q = -ORBIT_SPAN; q <= ORBIT_SPAN; ++q)
      for (int r = -ORBIT_SPAN; r <= ORBIT_SPAN; ++r) {
        const int d = std::max(std::abs(q), std::max(std::abs(r), std::abs(q + r)));
        orbit48[q + ORBIT_SPAN][r + ORBIT_SPAN] =
            (d >= 1 && d <= ORBIT_SPAN) ? (int)(std::lower_bound(all.begin(), all.end(), rep_of(q, r)) - all.begin())
                                        : -1;
      }
    for (int dq = -LEGAL_RADIUS; dq <= LEGAL_RADIUS; ++dq)
      for (int dr = -LEGAL_RADIUS; dr <= LEGAL_RADIUS; ++dr) {
        const int d = std::max(std::abs(dq), std::max(std::abs(dr), std::abs(dq + dr)));
        if (d < 1 || d > LEGAL_RADIUS) continue;
        disk_q.push_back(dq);
        disk_r.push_back(dr);
        disk_dist.push_back(d);
        disk_orbit.push_back(orbit48[dq + ORBIT_SPAN][dr + ORBIT_SPAN]);
        disk_on_axis.push_back(dq == 0 || dr == 0 || dq + dr == 0);
      }
  }
};

const Tables& tables() {
  static const Tables t;
  return t;
}

// ------------------------------------------------------------ hash table --
// int64 key -> int64 value, open addressing; insert keeps the first value.
class KeyMap {
 public:
  explicit KeyMap(size_t n) {
    size_t cap = 16;
    while (cap < 2 * n + 1) cap <<= 1;
    keys_.assign(cap, 0);
    vals_.assign(cap, -1);
    mask_ = cap - 1;
  }
  void insert(int64_t k, int64_t v) {
    for (size_t i = slot(k);; i = (i + 1) & mask_) {
      if (vals_[i] < 0) { keys_[i] = k; vals_[i] = v; return; }
      if (keys_[i] == k) return;
    }
  }
  int64_t find(int64_t k) const {
    for (size_t i = slot(k);; i = (i + 1) & mask_) {
      if (vals_[i] < 0) return -1;
      if (keys_[i] == k) return vals_[i];
    }
  }

 private:
  size_t slot(int64_t k) const { return (size_t)(((uint64_t)k * 0x9E3779B97F4A7C15ull) >> 17) & mask_; }
  std::vector<int64_t> keys_, vals_;
  size_t mask_;
};

// ------------------------------------------------------------- one position
struct Graph {
  int64_t n_s = 0, n_w = 0, n_l = 0, moves = 1;
  std::vector<int64_t> stone_qr, stone_own;
  std::vector<int64_t> window_feat, window_id;             // window_id: (axis, q, r) per window
  std::vector<int64_t> inc_stone, inc_window, inc_class;
  std::vector<int64_t> nearest;
  std::vector<int64_t> r_src, r_dst, r_orbit, r_own, r_axis;
  std::vector<int64_t> a_src, a_dst, a_axis;
  std::vector<int64_t> dec_cell, dec_window, dec_class;
  std::vector<int64_t> act_class, act_empty;               // act_empty: 3 per cell
  std::vector<float> tactical;                             // 11 per cell
};

struct PosIn {
  const int64_t* stone_qr;
  const int64_t* owner;
  int64_t n_s;
  int64_t mover;
  const int64_t* legal_qr;
  int64_t n_l;
  int64_t moves;
};

// Builds one position; returns an empty string or the refusal message.
std::string build_one(const PosIn& in, Graph& g) {
  const Tables& T = tables();
  if (in.n_l == 0) return "terminal position: the builder refuses it";
  if (in.moves != 1 && in.moves != 2)
    return "moves_remaining must be 1 or 2, got " + std::to_string(in.moves);
  const int64_t n_s = in.n_s, n_l = in.n_l;
  g.n_s = n_s;
  g.n_l = n_l;
  g.moves = in.moves;
  g.stone_qr.assign(in.stone_qr, in.stone_qr + 2 * n_s);
  g.stone_own.resize(n_s);
  for (int64_t i = 0; i < n_s; ++i) g.stone_own[i] = in.owner[i] != in.mover;

  // legal cells: packed key -> legal row (the first row holding that key)
  KeyMap legal(n_l);
  for (int64_t c = 0; c < n_l; ++c) legal.insert(pack(in.legal_qr[2 * c], in.legal_qr[2 * c + 1]), c);

  // ---- radius edges and nearest-stone distance (reference builder.py:427-460)
  const int nd = (int)T.disk_q.size();
  g.nearest.assign(n_l, n_s ? LEGAL_RADIUS + 1 : NEAREST_UNREACHED);
  if (n_s) {
    std::vector<int64_t> cnt(n_l + 1, 0);
    std::vector<int64_t> hit_c, hit_s;
    std::vector<int> hit_d;
    hit_c.reserve(n_s * 64); hit_s.reserve(n_s * 64); hit_d.reserve(n_s * 64);
    for (int64_t s = 0; s < n_s; ++s) {
      const int64_t q = in.stone_qr[2 * s], r = in.stone_qr[2 * s + 1];
      for (int d = 0; d < nd; ++d) {
        const int64_t c = legal.find(pack(q + T.disk_q[d], r + T.disk_r[d]));
        if (c < 0) continue;
        hit_c.push_back(c); hit_s.push_back(s); hit_d.push_back(d);
        ++cnt[c + 1];
        g.nearest[c] = std::min<int64_t>(g.nearest[c], T.disk_dist[d]);
      }
    }
    bool bad = false;
    for (int64_t c = 0; c < n_l && !bad; ++c) bad = g.nearest[c] > LEGAL_RADIUS;
    if (!bad) {
      KeyMap stones(n_s);
      for (int64_t s = 0; s < n_s; ++s) stones.insert(pack(in.stone_qr[2 * s], in.stone_qr[2 * s + 1]), s);
      for (int64_t c = 0; c < n_l && !bad; ++c) bad = stones.find(pack(in.legal_qr[2 * c], in.legal_qr[2 * c + 1])) >= 0;
    }
    if (bad) return "legal cells must be empty and within radius 8 of a stone";
    // stable counting sort by destination: sources stay ascending within a cell
    for (int64_t c = 0; c < n_l; ++c) cnt[c + 1] += cnt[c];
    const size_t ne = hit_c.size();
    g.r_src.resize(ne); g.r_dst.resize(ne); g.r_orbit.resize(ne); g.r_own.resize(ne); g.r_axis.resize(ne);
    std::vector<int64_t> at(cnt.begin(), cnt.end() - 1);
    for (size_t e = 0; e < ne; ++e) {
      const int64_t i = at[hit_c[e]]++;
      g.r_src[i] = hit_s[e];
      g.r_dst[i] = hit_c[e];
      g.r_orbit[i] = T.disk_orbit[hit_d[e]];
      g.r_own[i] = g.stone_own[hit_s[e]];
      g.r_axis[i] = T.disk_on_axis[hit_d[e]];
    }
  }

  // ---- directed distance-one neighbours among legal cells (builder.py:462-483)
  {
    static const int steps[6][2] = {{-1, 0}, {0, -1}, {-1, 1}, {1, 0}, {0, 1}, {1, -1}};
    std::vector<int64_t> cnt(n_l + 1, 0), hs, hd, ha;
    for (int64_t c = 0; c < n_l; ++c) {
      const int64_t q = in.legal_qr[2 * c], r = in.legal_qr[2 * c + 1];
      for (int j = 0; j < 6; ++j) {
        const int64_t dst = legal.find(pack(q + steps[j][0], r + steps[j][1]));
        if (dst < 0) continue;
        hs.push_back(c); hd.push_back(dst); ha.push_back(j % 3);
        ++cnt[dst + 1];
      }
    }
    for (int64_t c = 0; c < n_l; ++c) cnt[c + 1] += cnt[c];
    g.a_src.resize(hs.size()); g.a_dst.resize(hs.size()); g.a_axis.resize(hs.size());
    std::vector<int64_t> at(cnt.begin(), cnt.end() - 1);
    for (size_t e = 0; e < hs.size(); ++e) {
      const int64_t i = at[hd[e]]++;
      g.a_src[i] = hs[e]; g.a_dst[i] = hd[e]; g.a_axis[i] = ha[e];
    }
  }

  // ---- stones: duplicates refused (builder.py:567-570)
  KeyMap stones(n_s);
  {
    std::vector<int64_t> keys(n_s);
    for (int64_t s = 0; s < n_s; ++s) keys[s] = pack(in.stone_qr[2 * s], in.stone_qr[2 * s + 1]);
    std::vector<int64_t> sorted = keys;
    std::sort(sorted.begin(), sorted.end());
    if (std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end()) return "duplicate stone coordinates";
    for (int64_t s = 0; s < n_s; ++s) stones.insert(keys[s], s);
  }
  auto digit_at = [&](int64_t q, int64_t r) -> int {  // 0 empty, 1 own (mover's), 2 opponent's
    const int64_t s = stones.find(pack(q, r));
    return s < 0 ? 0 : 1 + (int)g.stone_own[s];
  };

  // ---- windows: every (axis, start) through a stone, ascending key (builder.py:572-585)
  struct Cand { int64_t key, q, r; int a; };
  std::vector<Cand> cand;
  cand.reserve(n_s * 3 * W);
  for (int64_t s = 0; s < n_s; ++s)
    for (int a = 0; a < 3; ++a)
      for (int k = 0; k < W; ++k) {
        const int64_t q = in.stone_qr[2 * s] - AX[a][0] * k, r = in.stone_qr[2 * s + 1] - AX[a][1] * k;
        cand.push_back({pack(q, r) * 4 + a, q, r, a});
      }
  std::sort(cand.begin(), cand.end(), [](const Cand& x, const Cand& y) { return x.key < y.key; });
  cand.erase(std::unique(cand.begin(), cand.end(), [](const Cand& x, const Cand& y) { return x.key == y.key; }),
             cand.end());
  const int64_t n_w = (int64_t)cand.size();
  g.n_w = n_w;
  KeyMap live(n_w);
  std::vector<int> pattern(n_w);
  g.window_feat.resize(n_w);
  g.window_id.resize(3 * n_w);
  for (int64_t w = 0; w < n_w; ++w) {
    const Cand& c = cand[w];
    live.insert(c.key, w);
    int pat = 0;
    for (int j = 0; j < W; ++j) {
      const int64_t q = c.q + AX[c.a][0] * j, r = c.r + AX[c.a][1] * j;
      const int64_t s = stones.find(pack(q, r));
      if (s < 0) continue;
      pat += (1 + (int)g.stone_own[s]) * T.pow3[j];
      g.inc_stone.push_back(s);
      g.inc_window.push_back(w);
      g.inc_class.push_back(j);  // slot for now; class once the pattern is known
    }
    pattern[w] = pat;
    g.window_feat[w] = T.rank[pat];
    g.window_id[3 * w] = c.a;
    g.window_id[3 * w + 1] = c.q;
    g.window_id[3 * w + 2] = c.r;
  }
  for (size_t e = 0; e < g.inc_class.size(); ++e) {
    const int cls = T.occ[pattern[g.inc_window[e]]][g.inc_class[e]];
    if (cls < 0) return "incidence entry pairs a window with a slot it does not occupy";
    g.inc_class[e] = cls;
  }

  // ---- decoder rows and action rows (builder.py:587-600, 292-424)
  g.act_empty.assign(3 * n_l, 0);
  g.tactical.assign(TACTICAL * n_l, 0.f);
  std::vector<int64_t> win_index(n_l * 3 * W);
  std::vector<int> own_c(n_l * 3 * W), opp_c(n_l * 3 * W);
  std::vector<char> five_mark(n_w, 0), four_mark(n_w, 0);
  int64_t five_remaining = 0, four_remaining = 0;
  for (int64_t c = 0; c < n_l; ++c) {
    const int64_t q0 = in.legal_qr[2 * c], r0 = in.legal_qr[2 * c + 1];
    for (int a = 0; a < 3; ++a) {
      int line[2 * W - 1];
      for (int o = 0; o < 2 * W - 1; ++o)
        line[o] = digit_at(q0 + AX[a][0] * (o - (W - 1)), r0 + AX[a][1] * (o - (W - 1)));
      if (line[W - 1] != 0) return "a legal action cell is occupied";
      for (int k = 0; k < W; ++k) {
        int pre = 0, own = 0, opp = 0;
        for (int j = 0; j < W; ++j) {
          const int d = line[j + (W - 1) - k];
          pre += d * T.pow3[j];
          own += d == 1;
          opp += d == 2;
        }
        const int64_t w = live.find(pack(q0 - AX[a][0] * k, r0 - AX[a][1] * k) * 4 + a);
        const int idx = (int)(c * 3 * W + a * W + k);
        win_index[idx] = w;
        own_c[idx] = own;
        opp_c[idx] = opp;
        const int post1 = T.post1[pre + T.pow3[k]][k];
        if (post1 < 0) return "a post-placement row lost its own stone";
        const bool kept = own > 0 || opp > 0;
        if ((w >= 0) != kept) return "the kept-window set disagrees with the action-row walk";
        if (kept) {
          const int cls = T.dec[pattern[w]][k];
          if (cls < 0) return "decoder entry pairs a window with a slot it already occupies";
          g.dec_cell.push_back(c);
          g.dec_window.push_back(w);
          g.dec_class.push_back(cls);
          g.act_class.push_back(post1);
          if (opp > 0 && own == 0) {
            if (opp == 5 && !five_mark[w]) { five_mark[w] = 1; ++five_remaining; }
            if (opp == 4 && !four_mark[w]) { four_mark[w] = 1; ++four_remaining; }
          }
        } else {
          ++g.act_empty[3 * c + T.slot_orbit[k]];
        }
      }
    }
  }
  const float rows_total = (float)(3 * W);
  const float five_f = (float)std::min<int64_t>(five_remaining, THREAT_CAP) / (float)THREAT_CAP;
  const float four_f = (float)std::min<int64_t>(four_remaining, THREAT_CAP) / (float)THREAT_CAP;
  for (int64_t c = 0; c < n_l; ++c) {
    int any_win = 0, max_own = 0, max_opp = 0, make5 = 0, make4 = 0, five_hit = 0, four_rows = 0, kept = 0;
    for (int i = 0; i < 3 * W; ++i) {
      const int own = own_c[c * 3 * W + i], opp = opp_c[c * 3 * W + i];
      max_own = std::max(max_own, own);
      max_opp = std::max(max_opp, opp);
      if (opp == 0 && own == W - 1) any_win = 1;
      if (opp == 0 && own + 1 == 5) ++make5;
      if (opp == 0 && own + 1 == 4) ++make4;
      if (opp > 0 && own == 0 && opp == 5) ++five_hit;
      if (opp > 0 && own == 0 && opp == 4) ++four_rows;
      kept += own > 0 || opp > 0;
    }
    float* t = &g.tactical[TACTICAL * c];
    t[0] = (float)any_win;
    t[1] = (float)(max_own + 1) / (float)W;
    t[2] = (float)max_opp / (float)W;
    t[3] = (float)make5 / rows_total;
    t[4] = (float)make4 / rows_total;
    t[5] = (float)five_hit / rows_total;
    t[6] = (float)four_rows / rows_total;
    t[7] = five_f;
    t[8] = four_f;
    t[9] = (float)(five_remaining > 0 && five_hit == five_remaining);
    t[10] = (float)kept / rows_total;
  }
  return std::string();
}

// Runs fn(i) for i in [0, n) over `threads` threads (0: hardware count).
template <typename F>
void parallel_for(int64_t n, int threads, F fn) {
  int t = threads > 0 ? threads : (int)std::thread::hardware_concurrency();
  if (t < 1) t = 1;
  if (t > n) t = (int)std::max<int64_t>(n, 1);
  if (t == 1) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<int64_t> next(0);
  std::vector<std::thread> pool;
  for (int k = 0; k < t; ++k)
    pool.emplace_back([&] {
      for (int64_t i; (i = next.fetch_add(1)) < n;) fn(i);
    });
  for (auto& th : pool) th.join();
}

}  // namespace enc
}  // namespace mb

struct mb_encoding {
  std::vector<mb::enc::Graph> graphs;
  // per-position offsets (n_pos + 1 each): stones, windows, incidences,
  // cells, radius edges, adjacency edges, decoder rows
  std::vector<int64_t> off[7];
  int64_t max_t = 0, max_w = 0, n_covered = 0;
};

extern "C" {

int mb_encode_positions(int64_t n_pos, const int64_t* stone_off, const int64_t* stone_qr, const int64_t* stone_owner,
                        const int64_t* mover, const int64_t* legal_off, const int64_t* legal_qr,
                        const int64_t* moves_remaining, int threads, mb_encoding** out) {
  using namespace mb::enc;
  MB_REQUIRE(out != nullptr, "encode_positions: null output handle");
  *out = nullptr;
  MB_REQUIRE(n_pos > 0, "empty batch");
  MB_REQUIRE(stone_off && legal_off && mover && moves_remaining, "encode_positions: null pointer");
  MB_REQUIRE(stone_off[0] == 0 && legal_off[0] == 0, "encode_positions: offsets must start at 0");
  for (int64_t i = 0; i < n_pos; ++i)
    MB_REQUIRE(stone_off[i + 1] >= stone_off[i] && legal_off[i + 1] >= legal_off[i],
               "encode_positions: offsets must be non-decreasing (position %lld)", (long long)i);
  MB_REQUIRE(stone_off[n_pos] == 0 || (stone_qr && stone_owner), "encode_positions: null stone arrays");
  MB_REQUIRE(legal_off[n_pos] == 0 || legal_qr, "encode_positions: null legal array");
  tables();  // built once, before the threads share it
  auto* e = new mb_encoding();
  e->graphs.resize(n_pos);
  std::vector<std::string> err(n_pos);
  parallel_for(n_pos, threads, [&](int64_t i) {
    PosIn in{stone_qr ? stone_qr + 2 * stone_off[i] : nullptr, stone_owner ? stone_owner + stone_off[i] : nullptr,
             stone_off[i + 1] - stone_off[i], mover[i], legal_qr ? legal_qr + 2 * legal_off[i] : nullptr,
             legal_off[i + 1] - legal_off[i], moves_remaining[i]};
    err[i] = build_one(in, e->graphs[i]);
  });
  for (int64_t i = 0; i < n_pos; ++i)
    if (!err[i].empty()) {
      delete e;
      return mb::fail(MB_INVALID_ARGUMENT, "position %lld: %s", (long long)i, err[i].c_str());
    }
  for (auto& o : e->off) o.assign(n_pos + 1, 0);
  int64_t max_s = 0, max_w = 0;
  for (int64_t i = 0; i < n_pos; ++i) {
    const Graph& g = e->graphs[i];
    const int64_t n[7] = {g.n_s, g.n_w, (int64_t)g.inc_stone.size(), g.n_l, (int64_t)g.r_src.size(),
                          (int64_t)g.a_src.size(), (int64_t)g.dec_cell.size()};
    for (int f = 0; f < 7; ++f) e->off[f][i + 1] = e->off[f][i] + n[f];
    max_s = std::max(max_s, g.n_s);
    max_w = std::max(max_w, g.n_w);
    // decoder rows are cell-major, so distinct cells are counted in one pass
    for (size_t r = 0; r < g.dec_cell.size(); ++r) e->n_covered += r == 0 || g.dec_cell[r] != g.dec_cell[r - 1];
  }
  e->max_t = max_s + GLOBAL_ROWS;
  e->max_w = max_w + 1;
  *out = e;
  return MB_OK;
}

int mb_encoding_sizes(const mb_encoding* e, int64_t* sizes) {
  MB_REQUIRE(e && sizes, "encoding_sizes: null pointer");
  const int64_t P = (int64_t)e->graphs.size();
  const int64_t v[MB_ENC_NSIZES] = {P, e->off[0][P], e->off[1][P], e->off[2][P], e->off[3][P], e->off[4][P],
                                    e->off[5][P], e->off[6][P], e->max_t, e->max_w, e->n_covered};
  std::memcpy(sizes, v, sizeof(v));
  return MB_OK;
}

int mb_encoding_fill(const mb_encoding* e, void* const* fields, int threads) {
  using namespace mb::enc;
  MB_REQUIRE(e && fields, "encoding_fill: null pointer");
  for (int f = 0; f < MB_ENC_NFIELDS; ++f) MB_REQUIRE(fields[f] != nullptr, "encoding_fill: field %d is null", f);
  const int64_t P = (int64_t)e->graphs.size();
  const auto& so = e->off[0];
  const auto& wo = e->off[1];
  const auto& io = e->off[2];
  const auto& co = e->off[3];
  const auto& ro = e->off[4];
  const auto& ao = e->off[5];
  const auto& dof = e->off[6];
  const int64_t max_t = e->max_t, max_w = e->max_w;
  auto L = [&](int f) { return static_cast<int64_t*>(fields[f]); };
  parallel_for(P, threads, [&](int64_t i) {
    const Graph& g = e->graphs[i];
    const int64_t s0 = so[i], w0 = wo[i], i0 = io[i], c0 = co[i], r0 = ro[i], a0 = ao[i], d0 = dof[i];
    for (int64_t s = 0; s < g.n_s; ++s) {
      L(MB_ENC_STONE_OWN)[s0 + s] = g.stone_own[s];
      L(MB_ENC_STONE_SLOT)[s0 + s] = i * max_t + GLOBAL_ROWS + s;
    }
    for (int64_t w = 0; w < g.n_w; ++w) {
      L(MB_ENC_WINDOW_FEAT)[w0 + w] = g.window_feat[w];
      for (int j = 0; j < 3; ++j) L(MB_ENC_WINDOW_ID)[3 * (w0 + w) + j] = g.window_id[3 * w + j];
      L(MB_ENC_WINDOW_SLOT)[w0 + w] = i * max_w + 1 + w;
    }
    L(MB_ENC_MOVES_IDX)[i] = g.moves - 1;
    for (size_t x = 0; x < g.inc_stone.size(); ++x) {
      L(MB_ENC_INC_STONE)[i0 + x] = g.inc_stone[x] + s0;
      L(MB_ENC_INC_WINDOW)[i0 + x] = g.inc_window[x] + w0;
      L(MB_ENC_INC_CLASS)[i0 + x] = g.inc_class[x];
    }
    int32_t* coords = static_cast<int32_t*>(fields[MB_ENC_COORDS]) + i * max_t * 2;
    uint8_t* attn = static_cast<uint8_t*>(fields[MB_ENC_ATTN_VALID]) + i * max_t;
    for (int64_t t = 0; t < max_t; ++t) {
      const int64_t s = t - GLOBAL_ROWS;
      const bool stone = s >= 0 && s < g.n_s;
      coords[2 * t] = stone ? (int32_t)g.stone_qr[2 * s] : 0;
      coords[2 * t + 1] = stone ? (int32_t)g.stone_qr[2 * s + 1] : 0;
      attn[t] = t < GLOBAL_ROWS || stone;
    }
    uint8_t* vv = static_cast<uint8_t*>(fields[MB_ENC_VALUE_VALID]) + i * max_w;
    for (int64_t t = 0; t < max_w; ++t) vv[t] = t == 0 || t <= g.n_w;
    L(MB_ENC_LEGAL_OFFSETS)[i] = c0;
    if (i == P - 1) L(MB_ENC_LEGAL_OFFSETS)[P] = co[P];
    for (int64_t c = 0; c < g.n_l; ++c) {
      L(MB_ENC_CELL_POS)[c0 + c] = i;
      L(MB_ENC_CELL_NEAREST)[c0 + c] = g.nearest[c];
      for (int j = 0; j < 3; ++j) L(MB_ENC_ACT_EMPTY)[3 * (c0 + c) + j] = g.act_empty[3 * c + j];
      std::memcpy(static_cast<float*>(fields[MB_ENC_ACT_TACTICAL]) + TACTICAL * (c0 + c), &g.tactical[TACTICAL * c],
                  TACTICAL * sizeof(float));
    }
    for (size_t x = 0; x < g.r_src.size(); ++x) {
      L(MB_ENC_RADIUS_SRC)[r0 + x] = g.r_src[x] + s0;
      L(MB_ENC_RADIUS_DST)[r0 + x] = g.r_dst[x] + c0;
      L(MB_ENC_RADIUS_ORBIT)[r0 + x] = g.r_orbit[x];
      L(MB_ENC_RADIUS_OWN)[r0 + x] = g.r_own[x];
      L(MB_ENC_RADIUS_ON_AXIS)[r0 + x] = g.r_axis[x];
    }
    for (size_t x = 0; x < g.a_src.size(); ++x) {
      L(MB_ENC_ADJ_SRC)[a0 + x] = g.a_src[x] + c0;
      L(MB_ENC_ADJ_DST)[a0 + x] = g.a_dst[x] + c0;
      L(MB_ENC_ADJ_AXIS)[a0 + x] = g.a_axis[x];
    }
    for (size_t x = 0; x < g.dec_cell.size(); ++x) {
      L(MB_ENC_DEC_CELL)[d0 + x] = g.dec_cell[x] + c0;
      L(MB_ENC_DEC_WINDOW)[d0 + x] = g.dec_window[x] + w0;
      L(MB_ENC_DEC_CLASS)[d0 + x] = g.dec_class[x];
      L(MB_ENC_ACT_CLASS)[d0 + x] = g.act_class[x];
    }
  });

  // Relay views and the action rows' window order (reference relay.py:48-94,
  // builder.py:840-878): stable counting sorts of the decoder rows. The rows
  // are already cell-major, so the cell-major view is the rows themselves.
  const int64_t n_d = dof[P], n_w = wo[P];
  const int64_t* dcell = L(MB_ENC_DEC_CELL);
  const int64_t* dwin = L(MB_ENC_DEC_WINDOW);
  const int64_t* dcls = L(MB_ENC_DEC_CLASS);
  int64_t* cell_ptr = L(MB_ENC_RELAY_CELL_PTR);
  std::vector<int64_t> edge_cell(n_d);
  int64_t nc = 0;
  for (int64_t r = 0; r < n_d; ++r) {
    if (r == 0 || dcell[r] != dcell[r - 1]) cell_ptr[nc++] = r;
    edge_cell[r] = nc - 1;
  }
  cell_ptr[nc] = n_d;
  std::memcpy(L(MB_ENC_RELAY_WINDOW), dwin, n_d * sizeof(int64_t));
  std::memcpy(L(MB_ENC_RELAY_CLASS), dcls, n_d * sizeof(int64_t));
  auto counting_sort = [&](const int64_t* key, int64_t n_keys, int64_t* ptr, int64_t* order) {
    std::fill(ptr, ptr + n_keys + 1, 0);
    for (int64_t r = 0; r < n_d; ++r) ++ptr[key[r] + 1];
    for (int64_t k = 0; k < n_keys; ++k) ptr[k + 1] += ptr[k];
    std::vector<int64_t> at(ptr, ptr + n_keys);
    for (int64_t r = 0; r < n_d; ++r) order[at[key[r]]++] = r;
  };
  int64_t* act_rev = L(MB_ENC_ACT_REV);
  counting_sort(dwin, n_w, L(MB_ENC_RELAY_WIN_PTR), act_rev);
  int64_t* wcell = L(MB_ENC_RELAY_WCELL);
  for (int64_t r = 0; r < n_d; ++r) wcell[r] = edge_cell[act_rev[r]];
  std::vector<int64_t> corder(n_d);
  counting_sort(dcls, DEC_CLASSES, L(MB_ENC_RELAY_CLS_PTR), corder.data());
  int64_t* ccell = L(MB_ENC_RELAY_CCELL);
  for (int64_t r = 0; r < n_d; ++r) ccell[r] = edge_cell[corder[r]];
  return MB_OK;
}

int mb_encoding_free(mb_encoding* e) {
  delete e;
  return MB_OK;
}

int mb_encoder_table(int which, int64_t* out, int64_t capacity) {
  using namespace mb::enc;
  const Tables& T = tables();
  std::vector<int64_t> v;
  switch (which) {
    case 0: for (int p = 0; p < NPAT; ++p) v.push_back(T.rank[p]); break;
    case 1: for (int p = 0; p < NPAT; ++p) for (int s = 0; s < W; ++s) v.push_back(T.occ[p][s]); break;
    case 2: for (int p = 0; p < NPAT; ++p) for (int s = 0; s < W; ++s) v.push_back(T.dec[p][s]); break;
    case 3: for (int p = 0; p < NPAT; ++p) for (int s = 0; s < W; ++s) v.push_back(T.post1[p][s]); break;
    case 4:
      for (int q = 0; q < 2 * ORBIT_SPAN + 1; ++q)
        for (int r = 0; r < 2 * ORBIT_SPAN + 1; ++r) v.push_back(T.orbit48[q][r]);
      break;
    default: return mb::fail(MB_INVALID_ARGUMENT, "encoder_table: unknown table %d", which);
  }
  MB_REQUIRE(out && capacity >= (int64_t)v.size(), "encoder_table: table %d needs %lld entries", which,
             (long long)v.size());
  std::copy(v.begin(), v.end(), out);
  return MB_OK;
}

}  // extern "C"
