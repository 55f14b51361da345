// Copy lists for forked sequences (fe_kv_fork_copies, fe_kv.h). Host code
// only: no device memory is touched, so it runs on a host without a GPU.
//
// The reference's BlockManager shares only whole published pages between
// sequences and never writes a published page (src/scheduler.cpp:6-29, the
// check at :27); the tokens of a prefix it cannot share are recomputed by a
// prefill. A fork that copies instead of recomputing needs, for every page
// of the shared prefix that the child does not share with the parent, one
// copy of the prefix tokens on that page from the parent's page to the
// child's. This file derives those copies from the two block tables, and
// rejects tables that would let one sequence write a page the other reads.
#include <stdint.h>

#include <string>
#include <unordered_set>

#include "fe_kv.h"

namespace fe {
int fail(int status, const std::string& msg);  // fe_kv_ops.cu: records fe_last_error()
}

extern "C" int fe_kv_fork_copies(int num_forks, const int32_t* parent_tables,
                                 const int32_t* parent_off, const int32_t* child_tables,
                                 const int32_t* child_off, const int64_t* fork_len, int page,
                                 int32_t* src, int32_t* dst, int32_t* ntok, int capacity,
                                 int* num_copies) {
  using fe::fail;
  if (num_copies) *num_copies = 0;
  if (num_forks < 0 || page <= 0 || capacity < 0 || !num_copies)
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_fork_copies: bad sizes");
  if (num_forks == 0) return FE_OK;
  if (!parent_tables || !parent_off || !child_tables || !child_off || !fork_len ||
      (capacity > 0 && (!src || !dst || !ntok)))
    return fail(FE_ERR_INVALID_ARGUMENT, "fe_kv_fork_copies: null pointer");
  int n = 0;
  for (int f = 0; f < num_forks; ++f) {
    const int32_t* parent = parent_tables + parent_off[f];
    const int32_t* child = child_tables + child_off[f];
    const int64_t np = int64_t(parent_off[f + 1]) - parent_off[f];
    const int64_t nc = int64_t(child_off[f + 1]) - child_off[f];
    const int64_t len = fork_len[f];
    const std::string at = "fe_kv_fork_copies: fork " + std::to_string(f) + ": ";
    if (np < 0 || nc < 0 || len < 0)
      return fail(FE_ERR_INVALID_ARGUMENT, at + "negative table size or fork length");
    const int64_t pages = (len + page - 1) / page;  // pages holding the shared prefix
    if (pages > np || pages > nc)
      return fail(FE_ERR_INVALID_ARGUMENT, at + "fork length beyond a block table");
    std::unordered_set<int32_t> parent_pages(parent, parent + np);
    for (int64_t j = 0; j < pages; ++j) {
      const int64_t tokens = len - j * page < page ? len - j * page : page;
      if (child[j] == parent[j]) {
        // a shared page must be full: both sequences append after `len`, so a
        // partial page would be written by one while the other reads it
        if (tokens < page)
          return fail(FE_ERR_INVALID_ARGUMENT,
                      at + "partial tail page " + std::to_string(parent[j]) +
                          " is shared; give the child a fresh page (copy-on-write)");
        continue;
      }
      if (child[j] < 0 || parent[j] < 0)
        return fail(FE_ERR_INVALID_ARGUMENT, at + "negative page id");
      if (parent_pages.count(child[j]))
        return fail(FE_ERR_INVALID_ARGUMENT,
                    at + "child page " + std::to_string(child[j]) +
                        " belongs to the parent at another position");
      if (n >= capacity)
        return fail(FE_ERR_CAPACITY, "fe_kv_fork_copies: more copies than `capacity`");
      src[n] = parent[j];
      dst[n] = child[j];
      ntok[n] = static_cast<int32_t>(tokens);
      ++n;
    }
    // beyond the prefix the child's pages are its own: none may be the parent's
    for (int64_t j = pages; j < nc; ++j)
      if (parent_pages.count(child[j]))
        return fail(FE_ERR_INVALID_ARGUMENT,
                    at + "child page " + std::to_string(child[j]) +
                        " past the fork belongs to the parent");
  }
  *num_copies = n;
  return FE_OK;
}
