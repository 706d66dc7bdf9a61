// Device-side state of the B200 GBDT training path.
//
// One tree is grown entirely from device-resident state.  Each iteration is
// four launches whose grids do not depend on any device value (partition ->
// histogram -> subtract+scan -> commit); every kernel reads what it needs (the
// batch of leaves being expanded, their ranges and splits, which histogram
// slots to fill) from `TreeState`, and the commit kernel lays out the next
// batch.  The host learns that a tree is done through mapped host memory.
//
// HBM layout (see the trainer for sizes):
//   bins_rm   uint8 [N][Fp]  row-major, Fp = F rounded up to 16 (histograms)
//   bins_cm   uint8 [F][N]   feature-major (partition reads one column)
//   rows[2]   int32 [N]      ping-pong row-id buffers; a leaf is a contiguous
//                            range [begin, begin+count) of one of them
//   pairs[2]  quantized (g,h) per row, kept in the same order as rows:
//             QUANT mode int16 (int8 g | uint8 h << 8), FIXED mode int2
//   hist      int32 [slots][F][3][B]  integer (g, h, count) cells per leaf,
//             then one work slot per batch item
//
// Reference map: the per-leaf histogram is gpu_active_rows.mojo:3903
// (_range_hist_atomic_kernel); the stable partition :1054-1707; sibling
// subtraction gpu_leaf_batching.mojo:1364 / histogram.mojo:3747; leaf batching
// gpu_leaf_batching.mojo:2438; the split scan split.mojo:601-1360 (restated in
// integer prefix sums, exact); leaf pick growth_policy.mojo:659-677; tree
// grower tree.mojo:3767-4256.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "mt_math.h"

namespace mtb {

constexpr int kMaxLeaves = 4096;
constexpr int kMaxNodes = 2 * kMaxLeaves - 1;

enum HistMode : int { MODE_FIXED = 1, MODE_QUANT = 2 };

struct SplitRec {
  double gain;
  int found;
  int feature;
  int bin;
  int default_left;
  int is_cat;
  int pad;
  long long n_left;
  unsigned long long bits[4];
};

constexpr int kMaxBatch = 32;                              // leaves expanded per iteration
// leaf records of one tree: 1 + 2 per expansion, expansions bounded by the
// histogram slots (2 * num_leaves + batch)
constexpr int kMaxPool = 4 * kMaxLeaves + 2 * kMaxBatch + 2;

// One leaf of the tree being grown (frontier leaves, speculative children).
struct LeafRec {
  int node;         // node id once the leaf is part of the tree, else -1
  int parent;       // leaf record of the parent, -1 for the root
  int buf;          // ping-pong row buffer holding the leaf's rows
  int hist_slot;    // histogram slot, -1 when none
  int state;        // 0 leaf, 1 expanded (children computed, split not committed), 2 split committed
  int child[2];     // leaf ids of the children once expanded
  int exp_buf;      // buffer holding this leaf's rows after its expansion
  long long begin;  // local range [begin, begin + count) in rows[buf]
  long long count;  // local rows (this device)
  long long gcount; // global rows (histogram count)
  double value;     // leaf output
  SplitRec split;   // best split; split.found == 0 when none
};

// One leaf expansion of the current iteration.
struct BatchItem {
  int leaf;           // leaf id being expanded
  int child[2];       // leaf ids of the left and right children
  int built_is_left;  // decided from global counts, identical on every device
  int work;           // work-slot index of the built child
  int built_hist;     // histogram slot of the built child
  int sib_hist;       // histogram slot of the derived child (= the parent's)
  int feature;
  int threshold;
  int default_left;
  int missing_bin;
  int is_cat;
  unsigned long long bits[4];
  int src_buf;
  int dst_buf;
  long long begin;    // parent local range
  long long count;
  long long tile0;    // first partition tile of this item
  unsigned long long cursor_left;   // local rows placed left (final = local n_left)
  unsigned long long cursor_right;  // local rows placed right
};

struct Batch {
  int n_items;
  int root;           // 1 for the root build (no partition; the child is the root itself)
  long long n_tiles;  // partition tiles over all items
  BatchItem items[kMaxBatch];
};

struct ChildTotals {
  long long g, h, c;
};

struct FeatBest {
  double gain;
  int bin;
  int flags;  // bit0 found, bit1 default_left, bit2 categorical
  long long n_left;  // global rows going left under this candidate
  unsigned long long bits[4];
};

// Feature-sharded data-parallel exchange: one rank's best split of a child
// over the features it owns, and the child's totals.
struct ChildRec {
  double gain;            // > 0 when found
  long long n_left;
  long long tg, th, tc;   // the child's totals (when has_totals)
  unsigned long long bits[4];
  int feature, bin, flags, found, has_totals, pad;
};

struct NodeRec {
  int feature;   // -1 for a leaf
  int thr;       // threshold bin, -1 for categorical and leaves
  int left;
  int right;
  int dleft;     // missing values go left
  int mbin;      // missing bin of the split feature, -1 when none
  int is_cat;
  int pad;
  unsigned long long bits[4];  // categorical set (bins going left)
  double value;
  double gain;
  long long count;  // global rows reaching the node
};

struct TreeHeader {
  int n_leaves;              // frontier size (= leaves of the committed tree)
  int n_nodes;
  int done;
  int error;
  unsigned int scan_ticket;  // blocks of the current scan launch that have finished
  int n_pool;                // leaf records used
  int n_hist;                // histogram slots used
  int iterations;            // expansion iterations run for this tree
  int n_table;               // entries of the final row -> leaf table
  int pick_steps;            // steps of the commit kernel's pick loops (real and simulated), summed
};

// Compact per-leaf view the commit kernel loads in one pass: the leaf's gain
// (-1 when it cannot split), whether its children are computed, and their ids.
struct LeafInfo {
  double gain;
  int child[2];
  int expanded;
  int pad;
};

struct TreeState {
  TreeHeader hdr;
  Batch batch;
  ChildTotals totals[2 * kMaxBatch];
  unsigned int child_done[2 * kMaxBatch];  // scan warps finished per child (reset by the folding warp)
  LeafInfo info[kMaxPool];
  int slot_leaf[kMaxLeaves];  // frontier slot -> leaf id
  LeafRec pool[kMaxPool];
  NodeRec nodes[kMaxNodes];
};

// Per-fit constants every kernel reads.
struct FitConst {
  long long n_rows;        // rows held by this device
  long long row_offset;    // global id of this device's first row
  int n_features;          // F
  int f_pad;               // Fp (row stride of bins_rm)
  int n_bins;              // B (histogram width)
  int mode;                // MODE_FIXED / MODE_QUANT
  int const_hess;          // hessian constant this fit (L2 unweighted)
  int num_leaves;
  int min_data_in_leaf;
  double lambda_l2;
  double lambda_l1;
  double min_child_hess;
  int max_cat_to_onehot;
  int max_cat_threshold;
  double cat_smooth;
  double cat_l2;
  int min_data_per_group;
  int quant_bins;
};

// Per-round scales (written on device by the scale kernel).
struct RoundScales {
  double g_total;   // FIXED: pairwise sum |g|;   QUANT: max |g|
  double h_total;
  float gsf, hsf;   // FIXED: pow2 scales as Float32
  double g_inv, h_inv;  // FIXED: 1 / scale (exact); QUANT: RN(1 / units)
  double g_units, h_units;  // QUANT: units per gradient / hessian
  double g_lim, h_lim;
  int hq_const;     // FIXED const-hessian per-row hessian units
  int wide;         // FIXED with the 2^52 bound and Int64 cells
  long long hq_const64;  // wide FIXED const-hessian per-row hessian units
};

}  // namespace mtb
