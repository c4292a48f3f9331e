// Step plan: the host turns one gc_step's work items into flat device arrays once per step; every kernel of the step
// reads them from one device buffer (uploaded with a single copy), so kernel arguments do not depend on the items'
// contents. Semantics follow abi/gc.h:139-157 and ref.py:90-112 of the reference:
//   token j of an item writes KV row pos + j (slot blocks[row / 16] * 16 + row % 16),
//   runs RoPE at position pos + depth(j),
//   attends to the list  [rows 0 .. pos-1] ++ [rows pos + a for a in path(j)]   (a chain: path(j) = 0..j).
// Attention walks that list in fixed 16-entry groups and fixed SPLIT-entry splits, whatever the batch holds, so a row's
// arithmetic is the same alone, in a batch, in a prefill chunk or as a tree node (batch invariance, abi/gc.h:146).
#pragma once
#include <stdint.h>

namespace gck {

constexpr int kBlock = 16;          // KV rows per block (page)
constexpr int kSplit = 512;         // attention list entries per split (32 groups of 16)
constexpr int kGroup = 16;          // attention list entries per MMA group

struct Item {                       // one gc_work
  int pos;                          // first KV row of token 0
  int ntok;
  int tok0;                         // index of token 0 among the step's tokens
  int blk_off;                      // offset of the block table in plan.blocks
  int nblk;
  int tree;                         // parents given
  int path_off;                     // tree: offset of token 0's path in plan.paths (paths of all tokens, concatenated)
  int pad;
};

struct QGroup {                     // up to 16/G consecutive chain tokens of one item, or one or two tree tokens
  int item;
  int j0;                           // first token (index within the item)
  int ntok;
  int nvis;                         // list length of the group's last token
  int nsplit;                       // ceil(nvis / split)
  int part_base;                    // partial slot of (head 0, split 0); (head h, split s) = base + h * nsplit + s
  int path_off;                     // tree token: its path (token indices within the item, root .. self) in plan.paths
  int path_len;                     // tree token: depth + 1; chain: 0
  int path_off1, path_len1;         // a second tree token j0 + 1 in the group (rows G .. 2G-1); path_len1 0: none
};

struct AttnWork {                   // one CTA of the attention kernel: nqg groups of one item, one kv head, one split
  int qg0;
  int nqg;
  int head;
  int split;
};

struct PlanView {                   // device pointers into the plan buffer
  const int *tok_id;                // [T]
  const int *rope_pos;              // [T]
  const int *kv_row;                // [T] physical row written by the token
  const int *first_tok;             // [T] step index of the token writing this row's page's first row, or -1
  const Item *items;                // [n_items]
  const QGroup *qgroups;            // [n_qg]
  const AttnWork *work;             // [n_work]
  const unsigned *blocks;           // block tables
  const int *paths;                 // tree paths
  const int *want_tok;              // [R] step index of each wanted row's token
  int T, n_items, n_qg, n_work, R, n_parts;
  int max_rows;                     // most query rows (tokens x G) of any query group
  int tree_cta;                     // 1: some attention CTA holds several tree nodes (private tail buffers needed)
  int split;                        // list entries per split: kSplit, or (tolerance buckets, few rows of work) a
                                    // shorter power of two, at least 64
};

}  // namespace gck
