// trace.cu -- FMT1 real-selection trace reader (host code).
//
// Reads the trace format written by the reference's capture tool
// (tools/capture_miss_trace.py:316-317, :368-370): a 40-byte header
// "FMT1", version 1, requests, steps, layers, page_tokens, block_tokens,
// kv_heads, head_dim, sel_pages (u32 little endian), then per (request, step,
// layer) a u16 count and that many u32 block ids (chained content hashes).
// Same checks as the reference reader (src/workloads/miss_trace.cuh:75-185):
// every header field must match the run, block_tokens == 4, page_tokens a
// multiple of it, count == sel_pages * blocks_per_page -- but a mismatch is
// reported as FERRY_E_INVAL with the reason instead of exiting the process.
// Raw ids are remapped to dense ids in first-seen order (global across
// requests, as the reference does at :136-145), and the largest per-request
// distinct-id count is returned as the slab capacity (:167, :174). The dense
// ids drive the device miss detector (ferry_lru_touch) exactly like the
// reference's LRU replay of the same trace.
#include <cstdio>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "common.cuh"

extern "C" int ferry_trace_load(const char* path, int requests, int steps, int layers,
                                int sel_blocks, int kv_heads, int head_dim, int64_t* blocks_out,
                                int64_t capacity, int64_t* unique_out, int32_t* slab_blocks_out) {
  using ferry::set_error;
  if (!path || requests < 1 || steps < 1 || layers < 1 || sel_blocks < 1 || !unique_out ||
      !slab_blocks_out)
    return set_error("trace_load: bad arguments"), FERRY_E_INVAL;
  const int64_t total = (int64_t)requests * steps * layers * sel_blocks;
  if (blocks_out && capacity < total)
    return set_error("trace_load: output holds %lld ids, the trace has %lld", (long long)capacity,
                     (long long)total),
           FERRY_E_INVAL;
  FILE* f = std::fopen(path, "rb");
  if (!f) return set_error("trace_load: cannot open %s", path), FERRY_E_INVAL;
  struct Closer {
    FILE* f;
    ~Closer() { std::fclose(f); }
  } closer{f};
  char magic[4];
  uint32_t h[9];
  if (std::fread(magic, 1, 4, f) != 4 || std::memcmp(magic, "FMT1", 4) != 0)
    return set_error("trace_load: %s: magic is not FMT1", path), FERRY_E_INVAL;
  if (std::fread(h, 4, 9, f) != 9) return set_error("trace_load: %s: truncated header", path), FERRY_E_INVAL;
  const uint32_t ver = h[0], R = h[1], S = h[2], L = h[3], PT = h[4], BT = h[5], KV = h[6], D = h[7],
                 SEL = h[8];
  if (ver != 1) return set_error("trace_load: %s: version %u is not 1", path, ver), FERRY_E_INVAL;
  if ((int)R != requests) return set_error("trace_load: num_requests %u != %d", R, requests), FERRY_E_INVAL;
  if ((int)S != steps) return set_error("trace_load: steps %u != %d", S, steps), FERRY_E_INVAL;
  if ((int)L != layers) return set_error("trace_load: layers %u != %d", L, layers), FERRY_E_INVAL;
  if ((int)KV != kv_heads) return set_error("trace_load: kv_heads %u != %d", KV, kv_heads), FERRY_E_INVAL;
  if ((int)D != head_dim) return set_error("trace_load: head_dim %u != %d", D, head_dim), FERRY_E_INVAL;
  if (BT != 4) return set_error("trace_load: block_tokens %u != 4", BT), FERRY_E_INVAL;
  if (PT % BT) return set_error("trace_load: page_tokens %u not a multiple of block_tokens", PT), FERRY_E_INVAL;
  if ((int)(SEL * (PT / BT)) != sel_blocks)
    return set_error("trace_load: sel_pages %u x blocks_per_page %u != sel_blocks %d", SEL, PT / BT,
                     sel_blocks),
           FERRY_E_INVAL;
  std::unordered_map<uint32_t, int64_t> idmap;
  std::vector<uint32_t> ids(sel_blocks);
  uint64_t max_per_req = 0;
  int64_t ev = 0;
  for (uint32_t r = 0; r < R; ++r) {
    std::unordered_set<uint32_t> raw_seen;
    for (uint32_t s = 0; s < S; ++s)
      for (uint32_t l = 0; l < L; ++l) {
        uint16_t cnt = 0;
        if (std::fread(&cnt, 2, 1, f) != 1)
          return set_error("trace_load: payload truncated (count at r=%u s=%u l=%u)", r, s, l), FERRY_E_INVAL;
        if ((int)cnt != sel_blocks)
          return set_error("trace_load: event (r=%u,s=%u,l=%u) selects %u blocks, expected %d", r, s, l,
                           (unsigned)cnt, sel_blocks),
                 FERRY_E_INVAL;
        if (std::fread(ids.data(), 4, cnt, f) != cnt)
          return set_error("trace_load: payload truncated (ids at r=%u s=%u l=%u)", r, s, l), FERRY_E_INVAL;
        for (int k = 0; k < (int)cnt; ++k) {
          const uint32_t raw = ids[k];
          raw_seen.insert(raw);
          auto it = idmap.find(raw);
          int64_t blk;
          if (it == idmap.end()) {
            blk = (int64_t)idmap.size();
            idmap.emplace(raw, blk);
          } else {
            blk = it->second;
          }
          if (blocks_out) blocks_out[ev] = blk;
          ++ev;
        }
      }
    if (raw_seen.size() > max_per_req) max_per_req = raw_seen.size();
  }
  *unique_out = (int64_t)idmap.size();
  *slab_blocks_out = (int32_t)max_per_req;
  return FERRY_OK;
}
