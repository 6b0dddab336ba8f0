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
// sorts, stable). Coordinate lookups read dense grids over the position's
// bounding box (hash tables keyed by the packed coordinate when the box is
// huge), so a position costs O(cells).
#include <algorithm>
#include <cstdint>
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

// Cell coordinate -> index. A dense grid over the position's bounding box
// (plus a margin covering every offset the builder looks at) when that box is
// modest, else the hash table above; lookups outside the box miss.
class CellIndex {
 public:
  CellIndex(int64_t q0, int64_t r0, int64_t nq, int64_t nr, bool dense, size_t n)
      : q0_(q0), r0_(r0), nq_(nq), nr_(nr), dense_(dense), map_(dense ? 0 : n) {
    if (dense_) grid_.assign((size_t)(nq * nr), -1);
  }
  void insert(int64_t q, int64_t r, int64_t v) {
    if (!dense_) { map_.insert(pack(q, r), v); return; }
    const int64_t dq = q - q0_, dr = r - r0_;
    if ((uint64_t)dq >= (uint64_t)nq_ || (uint64_t)dr >= (uint64_t)nr_) return;
    int32_t& g = grid_[(size_t)(dq * nr_ + dr)];
    if (g < 0) g = (int32_t)v;
  }
  int64_t find(int64_t q, int64_t r) const {
    if (!dense_) return map_.find(pack(q, r));
    const int64_t dq = q - q0_, dr = r - r0_;
    if ((uint64_t)dq >= (uint64_t)nq_ || (uint64_t)dr >= (uint64_t)nr_) return -1;
    return grid_[(size_t)(dq * nr_ + dr)];
  }
  // Dense grids only: the grid offset of a cell inside the box, the offset
  // step of a coordinate step, and the entry at an offset (no bounds check:
  // the caller keeps to the box).
  bool dense() const { return dense_; }
  int64_t offset(int64_t q, int64_t r) const { return (q - q0_) * nr_ + (r - r0_); }
  int64_t stride(int64_t dq, int64_t dr) const { return dq * nr_ + dr; }
  int64_t at(int64_t off) const { return grid_[(size_t)off]; }

 private:
  int64_t q0_, r0_, nq_, nr_;
  bool dense_;
  KeyMap map_;
  std::vector<int32_t> grid_;
};

// ------------------------------------------------------------- one position
// One position's rows in compact per-position form (local indices); the
// batch arrays are int64 and offset, written in phase 2.
struct RadiusEdge { int32_t src, dst; uint8_t orbit, own, on_axis; };
struct AdjEdge { int32_t src, dst; uint8_t axis; };
struct IncRow { int32_t stone, window; int16_t cls; };
struct DecRow { int32_t cell, window; int16_t cls, post1; };
struct Graph {
  int64_t n_s = 0, n_w = 0, n_l = 0, moves = 1;
  std::vector<int32_t> stone_qr;                            // as the int32 coords field stores them
  std::vector<uint8_t> stone_own;
  std::vector<int16_t> window_feat;
  std::vector<int64_t> window_id;                           // (axis, q, r) per window
  std::vector<IncRow> inc;
  std::vector<uint8_t> nearest;
  std::vector<RadiusEdge> radius;
  std::vector<AdjEdge> adj;
  std::vector<DecRow> dec;
  std::vector<uint8_t> act_empty;                           // 3 per cell
  std::vector<float> tactical;                              // 11 per cell
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
  if (in.n_l == 0) return "terminal position: no legal move left to evaluate";
  if (in.moves != 1 && in.moves != 2)
    return "a turn places one or two stones; got moves_remaining=" + std::to_string(in.moves);
  const int64_t n_s = in.n_s, n_l = in.n_l;
  g.n_s = n_s;
  g.n_l = n_l;
  g.moves = in.moves;
  g.stone_qr.resize(2 * n_s);
  for (int64_t i = 0; i < 2 * n_s; ++i) g.stone_qr[i] = (int32_t)in.stone_qr[i];
  g.stone_own.resize(n_s);
  for (int64_t i = 0; i < n_s; ++i) g.stone_own[i] = in.owner[i] != in.mover;

  // Bounding box of stones and legal cells, widened by the farthest offset
  // any lookup uses (distance 8 from a stone, 5 along a line, 1 to a
  // neighbour); a dense grid serves it when it holds at most 4M cells.
  int64_t qlo = INT64_MAX, qhi = INT64_MIN, rlo = INT64_MAX, rhi = INT64_MIN;
  auto widen = [&](const int64_t* qr, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
      qlo = std::min(qlo, qr[2 * i]); qhi = std::max(qhi, qr[2 * i]);
      rlo = std::min(rlo, qr[2 * i + 1]); rhi = std::max(rhi, qr[2 * i + 1]);
    }
  };
  widen(in.stone_qr, n_s);
  widen(in.legal_qr, n_l);
  constexpr int64_t MARGIN = LEGAL_RADIUS + 1;
  const bool bounded = qhi - qlo < (int64_t(1) << 20) && rhi - rlo < (int64_t(1) << 20) &&
                       qlo > -(int64_t(1) << 40) && rlo > -(int64_t(1) << 40) && qhi < (int64_t(1) << 40) &&
                       rhi < (int64_t(1) << 40);
  const int64_t nq = bounded ? qhi - qlo + 1 + 2 * MARGIN : 0, nr = bounded ? rhi - rlo + 1 + 2 * MARGIN : 0;
  const bool dense = bounded && nq * nr <= (int64_t(1) << 22);
  auto index = [&](size_t n) { return CellIndex(qlo - MARGIN, rlo - MARGIN, nq, nr, dense, n); };

  // legal cells: coordinate -> legal row (the first row holding that cell)
  CellIndex legal = index(n_l);
  for (int64_t c = 0; c < n_l; ++c) legal.insert(in.legal_qr[2 * c], in.legal_qr[2 * c + 1], c);

  // ---- radius edges and nearest-stone distance (reference builder.py:427-460)
  const int nd = (int)T.disk_q.size();
  g.nearest.assign(n_l, n_s ? LEGAL_RADIUS + 1 : NEAREST_UNREACHED);
  if (n_s) {
    std::vector<int32_t> cnt(n_l + 1, 0);
    struct Hit { int32_t c, s, d; };
    std::vector<Hit> hits;
    hits.reserve(n_s * T.disk_q.size());  // at most one hit per disk offset
    // dense box: each disk offset is one grid step (a stone's disk, radius
    // 8, stays inside the 9-cell margin)
    std::vector<int64_t> disk_off(dense ? nd : 0);
    for (int d = 0; d < (int)disk_off.size(); ++d) disk_off[d] = legal.stride(T.disk_q[d], T.disk_r[d]);
    for (int64_t s = 0; s < n_s; ++s) {
      const int64_t q = in.stone_qr[2 * s], r = in.stone_qr[2 * s + 1];
      const int64_t sbase = dense ? legal.offset(q, r) : 0;
      for (int d = 0; d < nd; ++d) {
        const int64_t c = dense ? legal.at(sbase + disk_off[d]) : legal.find(q + T.disk_q[d], r + T.disk_r[d]);
        if (c < 0) continue;
        hits.push_back({(int32_t)c, (int32_t)s, d});
        ++cnt[c + 1];
        g.nearest[c] = std::min<uint8_t>(g.nearest[c], (uint8_t)T.disk_dist[d]);
      }
    }
    bool bad = false;
    for (int64_t c = 0; c < n_l && !bad; ++c) bad = g.nearest[c] > LEGAL_RADIUS;
    if (!bad) {
      CellIndex stones = index(n_s);
      for (int64_t s = 0; s < n_s; ++s) stones.insert(in.stone_qr[2 * s], in.stone_qr[2 * s + 1], s);
      for (int64_t c = 0; c < n_l && !bad; ++c) bad = stones.find(in.legal_qr[2 * c], in.legal_qr[2 * c + 1]) >= 0;
    }
    if (bad) return "every legal cell must be empty and at most 8 steps from a stone";
    // stable counting sort by destination: sources stay ascending within a cell
    for (int64_t c = 0; c < n_l; ++c) cnt[c + 1] += cnt[c];
    g.radius.resize(hits.size());
    for (const Hit& h : hits)
      g.radius[cnt[h.c]++] = {h.s, h.c, (uint8_t)T.disk_orbit[h.d], g.stone_own[h.s], (uint8_t)T.disk_on_axis[h.d]};
  }

  // ---- directed distance-one neighbours among legal cells (builder.py:462-483)
  {
    static const int steps[6][2] = {{-1, 0}, {0, -1}, {-1, 1}, {1, 0}, {0, 1}, {1, -1}};
    std::vector<int32_t> cnt(n_l + 1, 0);
    std::vector<AdjEdge> hits;
    hits.reserve(6 * n_l);
    for (int64_t c = 0; c < n_l; ++c) {
      const int64_t q = in.legal_qr[2 * c], r = in.legal_qr[2 * c + 1];
      const int64_t cbase = dense ? legal.offset(q, r) : 0;
      for (int j = 0; j < 6; ++j) {
        const int64_t dst = dense ? legal.at(cbase + legal.stride(steps[j][0], steps[j][1]))
                                  : legal.find(q + steps[j][0], r + steps[j][1]);
        if (dst < 0) continue;
        hits.push_back({(int32_t)c, (int32_t)dst, (uint8_t)(j % 3)});
        ++cnt[dst + 1];
      }
    }
    for (int64_t c = 0; c < n_l; ++c) cnt[c + 1] += cnt[c];
    g.adj.resize(hits.size());
    for (const AdjEdge& h : hits) g.adj[cnt[h.dst]++] = h;
  }

  // ---- stones: duplicates refused (builder.py:567-570)
  CellIndex stones = index(n_s);
  {
    std::vector<int64_t> keys(n_s);
    for (int64_t s = 0; s < n_s; ++s) keys[s] = pack(in.stone_qr[2 * s], in.stone_qr[2 * s + 1]);
    std::sort(keys.begin(), keys.end());
    if (std::adjacent_find(keys.begin(), keys.end()) != keys.end()) return "two stones occupy the same cell";
    for (int64_t s = 0; s < n_s; ++s) stones.insert(in.stone_qr[2 * s], in.stone_qr[2 * s + 1], s);
  }
  auto digit_at = [&](int64_t q, int64_t r) -> int {  // 0 empty, 1 own (mover's), 2 opponent's
    const int64_t s = stones.find(q, r);
    return s < 0 ? 0 : 1 + (int)g.stone_own[s];
  };
  // With a dense box the digits sit in a grid of their own: a legal cell's
  // 11-cell line samples and window starts (at most 5 steps away, inside the
  // 9-cell margin) are then plain offsets from the cell's.
  std::vector<uint8_t> digit;
  if (dense) {
    digit.assign((size_t)(nq * nr), 0);
    for (int64_t s = 0; s < n_s; ++s)
      digit[(size_t)stones.offset(in.stone_qr[2 * s], in.stone_qr[2 * s + 1])] = (uint8_t)(1 + g.stone_own[s]);
  }

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
  CellIndex live[3] = {index(n_w), index(n_w), index(n_w)};  // window start -> window, per axis
  std::vector<int> pattern(n_w);
  g.window_feat.resize(n_w);
  g.window_id.resize(3 * n_w);
  for (int64_t w = 0; w < n_w; ++w) {
    const Cand& c = cand[w];
    live[c.a].insert(c.q, c.r, w);
    int pat = 0;
    for (int j = 0; j < W; ++j) {
      const int64_t q = c.q + AX[c.a][0] * j, r = c.r + AX[c.a][1] * j;
      const int64_t s = stones.find(q, r);
      if (s < 0) continue;
      pat += (1 + (int)g.stone_own[s]) * T.pow3[j];
      g.inc.push_back({(int32_t)s, (int32_t)w, (int16_t)j});  // slot for now; class once the pattern is known
    }
    pattern[w] = pat;
    g.window_feat[w] = (int16_t)T.rank[pat];
    g.window_id[3 * w] = c.a;
    g.window_id[3 * w + 1] = c.q;
    g.window_id[3 * w + 2] = c.r;
  }
  for (IncRow& e : g.inc) {
    const int cls = T.occ[pattern[e.window]][e.cls];
    if (cls < 0) return "internal: an occupied slot has no incidence class";
    e.cls = (int16_t)cls;
  }

  // ---- decoder rows and action rows (builder.py:587-600, 292-424)
  g.act_empty.assign(3 * n_l, 0);
  g.tactical.assign(TACTICAL * n_l, 0.f);
  g.dec.reserve(18 * n_l / 4 + 16);
  std::vector<uint8_t> five_hit(n_l, 0);
  std::vector<char> five_mark(n_w, 0), four_mark(n_w, 0);
  int64_t five_remaining = 0, four_remaining = 0;
  const float rows_total = (float)(3 * W);
  for (int64_t c = 0; c < n_l; ++c) {
    const int64_t q0 = in.legal_qr[2 * c], r0 = in.legal_qr[2 * c + 1];
    const int64_t base = dense ? stones.offset(q0, r0) : 0;
    int any_win = 0, max_own = 0, max_opp = 0, make5 = 0, make4 = 0, hit5 = 0, four_rows = 0, kept_rows = 0;
    for (int a = 0; a < 3; ++a) {
      int line[2 * W - 1];
      const int64_t step = dense ? stones.stride(AX[a][0], AX[a][1]) : 0;
      if (dense) {
        const uint8_t* d0 = digit.data() + base - step * (W - 1);
        for (int o = 0; o < 2 * W - 1; ++o) line[o] = d0[step * o];
      } else {
        for (int o = 0; o < 2 * W - 1; ++o)
          line[o] = digit_at(q0 + AX[a][0] * (o - (W - 1)), r0 + AX[a][1] * (o - (W - 1)));
      }
      if (line[W - 1] != 0) return "a legal cell holds a stone";
      // The window starting k steps before the cell covers line[5 - k ..
      // 10 - k]; its pattern and counts slide from k = 5 down to k = 0.
      int pre_k[W], own_k[W], opp_k[W];
      {
        int pre = 0, own = 0, opp = 0;
        for (int j = 0; j < W; ++j) {
          const int d = line[j];
          pre += d * T.pow3[j];
          own += d == 1;
          opp += d == 2;
        }
        for (int k = W - 1;; --k) {
          pre_k[k] = pre;
          own_k[k] = own;
          opp_k[k] = opp;
          if (k == 0) break;
          const int out = line[W - 1 - k], in = line[2 * W - 1 - k];
          pre = (pre - out) / 3 + in * T.pow3[W - 1];
          own += (in == 1) - (out == 1);
          opp += (in == 2) - (out == 2);
        }
      }
      for (int k = 0; k < W; ++k) {
        const int pre = pre_k[k], own = own_k[k], opp = opp_k[k];
        const int post1 = T.post1[pre + T.pow3[k]][k];
        if (post1 < 0) return "internal: a placement slot has no post-placement class";
        const bool kept = own > 0 || opp > 0;
        // only a row holding a stone can name a live window
        const int64_t w = !kept ? -1
                                : dense ? live[a].at(base - step * k)
                                        : live[a].find(q0 - AX[a][0] * k, r0 - AX[a][1] * k);
        if ((w >= 0) != kept) return "internal: a window through a stone is missing from the live set";
        max_own = std::max(max_own, own);
        max_opp = std::max(max_opp, opp);
        if (opp == 0 && own == W - 1) any_win = 1;
        if (opp == 0 && own + 1 == 5) ++make5;
        if (opp == 0 && own + 1 == 4) ++make4;
        if (kept) {
          const int cls = T.dec[pattern[w]][k];
          if (cls < 0) return "internal: an empty slot has no decoder class";
          g.dec.push_back({(int32_t)c, (int32_t)w, (int16_t)cls, (int16_t)post1});
          ++kept_rows;
          if (opp > 0 && own == 0) {
            if (opp == 5) {
              ++hit5;
              if (!five_mark[w]) { five_mark[w] = 1; ++five_remaining; }
            }
            if (opp == 4) {
              ++four_rows;
              if (!four_mark[w]) { four_mark[w] = 1; ++four_remaining; }
            }
          }
        } else {
          ++g.act_empty[3 * c + T.slot_orbit[k]];
        }
      }
    }
    float* t = &g.tactical[TACTICAL * c];
    t[0] = (float)any_win;
    t[1] = (float)(max_own + 1) / (float)W;
    t[2] = (float)max_opp / (float)W;
    t[3] = (float)make5 / rows_total;
    t[4] = (float)make4 / rows_total;
    t[5] = (float)hit5 / rows_total;
    t[6] = (float)four_rows / rows_total;
    t[10] = (float)kept_rows / rows_total;
    five_hit[c] = (uint8_t)hit5;
  }
  // the position-wide threat counts, known once every cell is walked
  const float five_f = (float)std::min<int64_t>(five_remaining, THREAT_CAP) / (float)THREAT_CAP;
  const float four_f = (float)std::min<int64_t>(four_remaining, THREAT_CAP) / (float)THREAT_CAP;
  for (int64_t c = 0; c < n_l; ++c) {
    float* t = &g.tactical[TACTICAL * c];
    t[7] = five_f;
    t[8] = four_f;
    t[9] = (float)(five_remaining > 0 && five_hit[c] == five_remaining);
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
  std::vector<int64_t> cov_off;  // covered (decoder-row) cells per position
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
  e->cov_off.assign(n_pos + 1, 0);
  int64_t max_s = 0, max_w = 0;
  for (int64_t i = 0; i < n_pos; ++i) {
    const Graph& g = e->graphs[i];
    const int64_t n[7] = {g.n_s, g.n_w, (int64_t)g.inc.size(), g.n_l, (int64_t)g.radius.size(),
                          (int64_t)g.adj.size(), (int64_t)g.dec.size()};
    for (int f = 0; f < 7; ++f) e->off[f][i + 1] = e->off[f][i] + n[f];
    max_s = std::max(max_s, g.n_s);
    max_w = std::max(max_w, g.n_w);
    // decoder rows are cell-major, so distinct cells are counted in one pass
    int64_t cov = 0;
    for (size_t r = 0; r < g.dec.size(); ++r) cov += r == 0 || g.dec[r].cell != g.dec[r - 1].cell;
    e->cov_off[i + 1] = e->cov_off[i] + cov;
  }
  e->n_covered = e->cov_off[n_pos];
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

}  // extern "C"

// The collated arrays with index fields of type T (int64, or int32 for
// the narrow layout whose host-to-device copy is half the size).
template <typename T>
static int encoding_fill(const mb_encoding* e, void* const* fields, int threads) {
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
  auto L = [&](int f) { return static_cast<T*>(fields[f]); };
  std::vector<int32_t> cls_hist((size_t)P * DEC_CLASSES, 0);
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
    for (size_t x = 0; x < g.inc.size(); ++x) {
      L(MB_ENC_INC_STONE)[i0 + x] = g.inc[x].stone + s0;
      L(MB_ENC_INC_WINDOW)[i0 + x] = g.inc[x].window + w0;
      L(MB_ENC_INC_CLASS)[i0 + x] = g.inc[x].cls;
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
    for (size_t x = 0; x < g.radius.size(); ++x) {
      const RadiusEdge& r = g.radius[x];
      L(MB_ENC_RADIUS_SRC)[r0 + x] = r.src + s0;
      L(MB_ENC_RADIUS_DST)[r0 + x] = r.dst + c0;
      L(MB_ENC_RADIUS_ORBIT)[r0 + x] = r.orbit;
      L(MB_ENC_RADIUS_OWN)[r0 + x] = r.own;
      L(MB_ENC_RADIUS_ON_AXIS)[r0 + x] = r.on_axis;
    }
    for (size_t x = 0; x < g.adj.size(); ++x) {
      L(MB_ENC_ADJ_SRC)[a0 + x] = g.adj[x].src + c0;
      L(MB_ENC_ADJ_DST)[a0 + x] = g.adj[x].dst + c0;
      L(MB_ENC_ADJ_AXIS)[a0 + x] = g.adj[x].axis;
    }
    for (size_t x = 0; x < g.dec.size(); ++x) {
      const DecRow& d = g.dec[x];
      L(MB_ENC_DEC_CELL)[d0 + x] = d.cell + c0;
      L(MB_ENC_DEC_WINDOW)[d0 + x] = d.window + w0;
      L(MB_ENC_DEC_CLASS)[d0 + x] = d.cls;
      L(MB_ENC_ACT_CLASS)[d0 + x] = d.post1;
      L(MB_ENC_RELAY_WINDOW)[d0 + x] = d.window + w0;
      L(MB_ENC_RELAY_CLASS)[d0 + x] = d.cls;
    }
    // Relay views of this position's rows (reference relay.py:48-94): rows
    // are cell-major already, so cell runs are read off directly; the window
    // view is a counting sort within the position, because a position's
    // windows and rows both form one contiguous block. Class counts feed the
    // batch-wide class view below.
    const int64_t k0 = e->cov_off[i];
    T* cell_ptr = L(MB_ENC_RELAY_CELL_PTR);
    const size_t nd = g.dec.size();
    std::vector<int64_t> ecell(nd);
    int64_t k = k0 - 1;
    for (size_t x = 0; x < nd; ++x) {
      if (x == 0 || g.dec[x].cell != g.dec[x - 1].cell) cell_ptr[++k] = d0 + (int64_t)x;
      ecell[x] = k;
    }
    T* win_ptr = L(MB_ENC_RELAY_WIN_PTR) + w0;
    std::vector<int64_t> at(g.n_w + 1, 0);
    for (size_t x = 0; x < nd; ++x) ++at[g.dec[x].window + 1];
    for (int64_t w = 0; w < g.n_w; ++w) at[w + 1] += at[w];
    for (int64_t w = 0; w < g.n_w; ++w) win_ptr[w] = d0 + at[w];
    for (size_t x = 0; x < nd; ++x) {
      const int64_t pos = d0 + at[g.dec[x].window]++;
      L(MB_ENC_ACT_REV)[pos] = d0 + (int64_t)x;
      L(MB_ENC_RELAY_WCELL)[pos] = ecell[x];
    }
    int32_t* h = &cls_hist[(size_t)i * DEC_CLASSES];
    for (size_t x = 0; x < nd; ++x) ++h[g.dec[x].cls];
  });

  // Batch-wide ends of the relay views, then the class view: a stable
  // counting sort whose per-(class, position) starts come from the counts,
  // so each position scatters its own rows.
  const int64_t n_d = dof[P], n_w = wo[P];
  L(MB_ENC_RELAY_CELL_PTR)[e->n_covered] = n_d;
  L(MB_ENC_RELAY_WIN_PTR)[n_w] = n_d;
  T* cls_ptr = L(MB_ENC_RELAY_CLS_PTR);
  std::vector<int64_t> start((size_t)P * DEC_CLASSES);
  int64_t run = 0;
  for (int c = 0; c < DEC_CLASSES; ++c) {
    cls_ptr[c] = run;
    for (int64_t i = 0; i < P; ++i) {
      start[(size_t)i * DEC_CLASSES + c] = run;
      run += cls_hist[(size_t)i * DEC_CLASSES + c];
    }
  }
  cls_ptr[DEC_CLASSES] = run;
  parallel_for(P, threads, [&](int64_t i) {
    const Graph& g = e->graphs[i];
    int64_t* st = &start[(size_t)i * DEC_CLASSES];
    int64_t k = e->cov_off[i] - 1;
    for (size_t x = 0; x < g.dec.size(); ++x) {
      if (x == 0 || g.dec[x].cell != g.dec[x - 1].cell) ++k;
      L(MB_ENC_RELAY_CCELL)[st[g.dec[x].cls]++] = k;
    }
  });
  return MB_OK;
}

extern "C" {

int mb_encoding_fill(const mb_encoding* e, void* const* fields, int threads) {
  return encoding_fill<int64_t>(e, fields, threads);
}

int mb_encoding_fill_narrow(const mb_encoding* e, void* const* fields, int threads) {
  MB_REQUIRE(e, "encoding_fill_narrow: null encoding");
  int64_t sizes[11];
  const int st = mb_encoding_sizes(e, sizes);
  if (st != MB_OK) return st;
  for (int i = 0; i < 11; ++i)
    MB_REQUIRE(sizes[i] < INT32_MAX, "encoding_fill_narrow: %lld entries do not fit int32 indices", (long long)sizes[i]);
  return encoding_fill<int32_t>(e, fields, threads);
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
