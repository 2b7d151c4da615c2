// Where a KV cache keeps (cache row, KV head, position) within one layer's K or V.
#pragma once

#include <stdint.h>

namespace qi {

// Packed (table == nullptr): the reference's layout, one head of one row a contiguous run
// of max_len positions: element (row, head, pos) at ((row * 2 + head) * max_len + pos) * 64.
// Paged: pages of `page` positions of one row, both heads per page; table[row * ppr +
// pos / page] is the page of (row, pos) (-1: unmapped), element at
// ((page_id * 2 + head) * page + pos % page) * 64. Pages hold a multiple of 128 positions,
// so a 128-key attention tile never straddles two pages.
struct KvLayout {
  const int32_t* table;
  int page;
  int ppr;
  int n_pages;
};

}  // namespace qi
