// attn_decode.cu -- host side of the split-K decode: batch planning
// (plan_decode), workspace layout and the C ABI entry points.  The kernels
// and their launcher template live in attn_decode_kern.cuh; the launcher is
// instantiated per V format and score path in attn_decode_v*.cu.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "attn_decode_kern.cuh"

namespace g9 {
extern template cudaError_t launch_decode_t<1, 0, false>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<2, 0, false>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<1, 0, true>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<2, 0, true>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<1, 1, false>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<2, 1, false>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<1, 1, true>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<2, 1, true>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<1, 2, false>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<2, 2, false>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<1, 2, true>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<2, 2, true>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<1, 3, false>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<2, 3, false>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<1, 3, true>(const DecodeParams&, cudaStream_t);
extern template cudaError_t launch_decode_t<2, 3, true>(const DecodeParams&, cudaStream_t);

static int pad_odd16(int bytes) {
  int s = (bytes + 15) & ~15;
  if (((s / 16) & 1) == 0) s += 16;
  return s;
}

// Key order of the transposed consumer: per quad of 4 keys, which two feed
// k-slots (2j, 2j+1).  Chosen to minimise shared-memory wavefronts of the K
// fragment loads (8 rows x 4 lanes per instruction, 2-byte loads) for the
// launch's K row addresses.
// vgs > 0: 16-bit V rows in vgt-token groups (vgs bytes, rows hgb_v apart),
// read by ldmatrix.trans 8 keys at a time; their 16-byte rows should fall in
// 8 different bank groups as well.
static uint32_t search_tr_table(int kgs, int hgb_k, int vgs, int hgb_v, int vgt) {
  using namespace dec;
  auto kaddr = [&](int key) { return (key >> 2) * kgs + (key & 3) * hgb_k; };
  auto vaddr = [&](int key) { return (key / vgt) * vgs + (key % vgt) * hgb_v; };
  static const int pairs[6][4] = {{0, 1, 2, 3}, {0, 2, 1, 3}, {0, 3, 1, 2}, {1, 2, 0, 3}, {1, 3, 0, 2}, {2, 3, 0, 1}};
  auto wavefronts = [](const int* addr, int n) {   // 4-byte banks; same word is a broadcast
    int words[32][32], cnt[32] = {0}, worst = 0;
    for (int i = 0; i < n; ++i) {
      const int w = addr[i] >> 2, b = w & 31;
      bool seen = false;
      for (int k = 0; k < cnt[b]; ++k) seen |= words[b][k] == w;
      if (!seen) words[b][cnt[b]++] = w;
      worst = std::max(worst, cnt[b]);
    }
    return worst;
  };
  uint32_t best = 0;
  int best_cost = 1 << 30;
  for (int c = 0; c < 6 * 6 * 6 * 6; ++c) {
    int sel[4], cc = c;
    for (int q = 0; q < 4; ++q) { sel[q] = cc % 6; cc /= 6; }
    int cost = 0;
    for (int half = 0; half < 2; ++half) {
      int rows[8];
      for (int rq = 0; rq < 8; ++rq) {
        const int q = rq >> 1;
        rows[rq] = kaddr(4 * q + pairs[sel[q]][2 * half + (rq & 1)]);
      }
      for (int blk = 0; blk < 4; ++blk) {
        int a[32];
        for (int i = 0; i < 4; ++i) {
          for (int l = 0; l < 32; ++l) a[l] = rows[l >> 2] + blk * QBLOCK + 2 + 2 * (l & 3) + 8 * i;
          cost += wavefronts(a, 32);
        }
        for (int l = 0; l < 32; ++l) a[l] = rows[l >> 2] + blk * QBLOCK;
        cost += wavefronts(a, 32);
      }
      if (vgs > 0) {      // 16 ldmatrix phases per page and half
        int cnt[8] = {0}, worst = 0;
        for (int rq = 0; rq < 8; ++rq) {
          const int q = rq >> 1;
          const int g = (vaddr(4 * q + pairs[sel[q]][2 * half + (rq & 1)]) >> 4) & 7;
          worst = std::max(worst, ++cnt[g]);
        }
        cost += 16 * worst;
      }
    }
    if (cost < best_cost) {
      best_cost = cost;
      best = 0;
      for (int q = 0; q < 4; ++q) {
        const int* pr = pairs[sel[q]];
        best |= (uint32_t)(pr[0] | (pr[1] << 2) | (pr[2] << 4) | (pr[3] << 6)) << (8 * q);
      }
    }
  }
  return best;
}

// The search depends only on the K row geometry; results are cached (a few
// layouts per process).
static uint32_t choose_tr_table(const DecodeParams& d) {
  struct Entry { int kgs, hgb_k, vgs, hgb_v, vgt; uint32_t tab; };
  static Entry cache[16];
  static int n = 0;
  static std::mutex mu;
  const int hgb_k = d.HG * d.rb_k;
  const bool v16 = d.p.v_fmt == G9_VFMT_F16 || d.p.v_fmt == G9_VFMT_BF16;
  const int vgs = v16 ? d.vgs : 0, hgb_v = v16 ? d.HG * d.rb_v : 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (cache[i].kgs == d.kgs && cache[i].hgb_k == hgb_k && cache[i].vgs == vgs && cache[i].hgb_v == hgb_v &&
        cache[i].vgt == d.vgt)
      return cache[i].tab;
  const uint32_t tab = search_tr_table(d.kgs, hgb_k, vgs, hgb_v, d.vgt);
  if (n < 16) cache[n++] = Entry{d.kgs, hgb_k, vgs, hgb_v, d.vgt, tab};
  return tab;
}

static bool decode_tr_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GFX906_FA_DECODE_TRANSPOSED");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Most query rows per kv head (n_q * G) a sequence may have to be handled by
// the decode kernel; longer ones go to the prefill kernel.  24 when the
// transposed consumer (up to three 8-row n-tiles) serves the batch, else 32
// (two 16-row m-tiles).  The dispatcher and plan_decode both use it.
int decode_row_cap(const G9AttnBatch& p) {
  const int G = p.num_heads_kv > 0 ? p.num_heads_q / p.num_heads_kv : 0;
  const int HG = p.num_heads_kv % 8 == 0 ? 8 : (p.num_heads_kv % 4 == 0 ? 4 : (p.num_heads_kv % 2 == 0 ? 2 : 1));
  const bool tr = (p.v_fmt == G9_VFMT_Q8T || p.v_fmt == G9_VFMT_F16 || p.v_fmt == G9_VFMT_BF16) && G >= 1 && G <= 24 && p.num_heads_kv > 0 &&
                  (int64_t)p.num_seqs * (p.num_heads_kv / HG) <= dec::kMaxRanksTR && decode_tr_enabled();
  return tr ? 24 : 32;
}

// Fills DecodeParams from the batch; returns cudaErrorInvalidValue when the
// batch is outside what the decode kernel handles.
static cudaError_t plan_decode(const G9AttnBatch& p, DecodeParams& d, int& mt) {
  using namespace dec;
  if (p.head_dim != D || p.block_size != PAGE) return cudaErrorInvalidValue;
  if (p.num_seqs < 0 || p.num_heads_kv <= 0 || p.num_heads_q <= 0 || p.num_heads_q % p.num_heads_kv)
    return cudaErrorInvalidValue;
  if (p.seq_q < 0 || p.max_kv < 0 || p.max_blocks < 0) return cudaErrorInvalidValue;
  if (p.q_dtype < 0 || p.q_dtype > 2 || p.out_dtype < 0 || p.out_dtype > 3 || p.v_fmt < 0 || p.v_fmt > 3)
    return cudaErrorInvalidValue;
  if (p.out_dtype == G9_DT_FP8E4M3 && !p.out_scale) return cudaErrorInvalidValue;
  // Q rows are read as pairs of elements (8-byte fp32 / 4-byte 16-bit loads)
  if (((uintptr_t)p.q & 7) || (p.q_seq_stride | p.q_tok_stride | p.q_head_stride) & 1) return cudaErrorInvalidValue;
  d = DecodeParams{};
  d.p = p;
  d.G = p.num_heads_q / p.num_heads_kv;
  const int R = std::min(d.G * std::max(p.seq_q, 1), decode_row_cap(p));
  mt = R <= 16 ? 1 : 2;
  d.max_rows = R;
  d.R_pad = 16 * mt;
  const int Hkv = p.num_heads_kv;
  d.HG = Hkv % 8 == 0 ? 8 : (Hkv % 4 == 0 ? 4 : (Hkv % 2 == 0 ? 2 : 1));
  if (Hkv > 8 && d.HG != 8) return cudaErrorInvalidValue;
  d.HGN = Hkv / d.HG;
  d.ppw = 1;
  d.P = NWC / d.HG;                        // one page per group per stage (PPW = 1)
  d.rb_k = q8_row_bytes(D);
  const bool vq8t = p.v_fmt == G9_VFMT_Q8T;
  d.rb_v = (p.v_fmt == G9_VFMT_Q8 || vq8t) ? q8_row_bytes(D) : 2 * D;
  // dense pages: the rows of one token (all heads) are contiguous
  if (p.k_head_stride != d.rb_k || p.k_tok_stride != (int64_t)Hkv * d.rb_k) return cudaErrorInvalidValue;
  if (!vq8t && (p.v_head_stride != d.rb_v || p.v_tok_stride != (int64_t)Hkv * d.rb_v)) return cudaErrorInvalidValue;
  d.vrec = PAGE * d.rb_v;                 // page-transposed record (2176 bytes)
  if (vq8t && (p.v_head_stride < d.vrec || p.v_head_stride % 16)) return cudaErrorInvalidValue;
  d.vrec_contig = vq8t && p.v_head_stride == d.vrec;
  // Shared-memory layout per page: K in 4 groups of 4 tokens, V in 8 groups of
  // 2 tokens, each group padded to an odd multiple of 16 bytes.  When the
  // row groups of consecutive tokens are adjacent in HBM (all kv heads in one
  // CTA) a group is one bulk copy, else one copy per token.  Copies need
  // 16-byte aligned sources and sizes.
  const int hgk = d.HG * d.rb_k, hgv = d.HG * d.rb_v;
  d.contig = p.k_tok_stride == hgk && (vq8t || p.v_tok_stride == hgv);
  if (((uintptr_t)p.k_cache | (uintptr_t)p.v_cache | (uintptr_t)p.k_page_stride | (uintptr_t)p.v_page_stride) & 15)
    return cudaErrorInvalidValue;
  // head groups after the first start at h0 = z*HG heads into a token's rows
  if (d.HGN > 1 && (((int64_t)d.HG * p.k_head_stride) % 16 || (!vq8t && ((int64_t)d.HG * p.v_head_stride) % 16)))
    return cudaErrorInvalidValue;
  if (d.contig) {
    if ((2 * hgk) % 16 || (!vq8t && (2 * hgv) % 16)) return cudaErrorInvalidValue;
  } else {
    if (hgk % 16 || p.k_tok_stride % 16) return cudaErrorInvalidValue;
    if (!vq8t && (hgv % 16 || p.v_tok_stride % 16)) return cudaErrorInvalidValue;
  }
  d.kgs = pad_odd16(4 * hgk);
  // Up to four kv heads per CTA the copy-request rate of the producer binds
  // (per request cost, not bytes), so a page's K rows (adjacent in HBM) are
  // copied whole into an unpadded page.  At one or two heads the padded
  // 4-token groups remove no bank conflicts anyway (1.5 / 2 wavefronts per
  // fragment load either way); at four the padding would halve them, but the
  // fewer copies win (config 3's four-head share: Q8_0 V 211 -> 182 us, fp16 V
  // 318 -> 292 us).  At eight heads the padded 4-token groups stay (whole-page
  // copies: Q8_0 V 351 -> 437 us).
  d.kwhole = d.contig && d.HG <= 4;
  if (const char* e = std::getenv("GFX906_FA_DECODE_KWHOLE"))      // tuning override: whole-page K copies
    d.kwhole = d.contig && std::atoi(e) != 0;
  if (d.kwhole) d.kgs = 4 * hgk;
  d.nranks = p.num_seqs * d.HGN;
  // transposed consumer: up to 3 n-tiles of 8 query rows; 16 compute warps
  // only for one n-tile and one kv head per CTA (register budget)
  d.nt = (R + 7) / 8;
  const bool v16 = p.v_fmt == G9_VFMT_F16 || p.v_fmt == G9_VFMT_BF16;
  // Every transposed batch runs 8 compute warps; at one kv head per CTA each
  // warp takes two pages per stage (16 pages, below), measured 62.7 us
  // against 70.3 us for 16 warps of one page each on config 3's one-head
  // share (the 16-warp geometry spills at its 104-register budget).
  // GFX906_FA_DECODE_TRW=16 selects that geometry (tuning override).
  d.tr = (vq8t || v16) && R <= 24 && d.nranks <= kMaxRanksTR && decode_tr_enabled() ? NWC : 0;
  if (d.tr && vq8t && d.HG == 1 && d.nt == 1) {
    const char* e = std::getenv("GFX906_FA_DECODE_TRW");
    if (e && std::atoi(e) == NWC_TR) d.tr = NWC_TR;
  }
  // 16-bit V tokens per shared-memory group (one copy per group when rows are
  // adjacent): 2, padded, for the 16-row kernel; the transposed kernel takes
  // larger groups (fewer copy requests; its key order keeps the ldmatrix
  // reads spread over the banks as far as the layout allows)
  d.vgt = 2;
  if (d.tr && v16 && d.contig) d.vgt = d.HG <= 2 ? kVgtSmallHG : kVgtLargeHG;
  if (const char* e = std::getenv("GFX906_FA_DECODE_VGT")) {      // tuning override
    const int v = std::atoi(e);
    if (d.tr && v16 && d.contig && (v == 2 || v == 4 || v == 8 || v == 16)) d.vgt = v;
  }
  {
    const int kc = d.kwhole ? 1 : (d.contig ? 4 : 16);
    const int vc = vq8t ? (d.vrec_contig ? 1 : d.HG) : (d.contig ? PAGE / d.vgt : 16);
    int l = 1;
    while ((1 << l) < kc + vc) ++l;
    d.cps_log2 = l;                       // 2 .. 32 slots
  }
  d.vgs = pad_odd16(d.vgt * hgv);
  d.kpage = (PAGE / 4) * d.kgs;
  // page-transposed V: the HG records back to back (ldmatrix rows are 16
  // consecutive bytes, conflict-free at any 16-byte aligned base)
  d.vpage = vq8t ? d.HG * d.vrec : (PAGE / d.vgt) * d.vgs;
  const int nwc = d.tr ? d.tr : NWC;
  d.P = nwc / d.HG;
  d.NG = nwc / d.HG;
  const int q_bytes = mt == 2 && !d.tr ? NWC * mt * 16 * QROW : 0;   // one Q tile per compute warp
  const int cpre_bytes = (d.tr ? ((d.nranks + 1) * 4 + 15) & ~15 : 0) + (d.tr && d.nt >= 3 ? NWC * (24 * QROW + 512) : 0);
  constexpr int64_t kSmem = 227 * 1024;
  auto need = [&](int nst, int pages) {
    return (int64_t)nst * pages * (d.kpage + d.vpage) + q_bytes + cpre_bytes;
  };
  // Two pages per warp and stage give each warp two independent streams of
  // loads / conversions / MMAs (the kernel is latency-bound), with 3 stages
  // (one m-tile only: with two the registers would spill); else one page per
  // warp with 4 stages, or 3 when 4 do not fit.
  // 16-bit V rows: two pages per warp too, in two stages when three do not
  // fit (config 3 with fp16 V: two-head share 177.5 -> 151.8 us, one head
  // 110.7 -> 106.8 us; four heads 287 -> 249 us, all eight 514 -> 465 us);
  // GFX906_FA_DECODE_V16PPW2=0 turns it off (tuning override).
  const char* v16p = std::getenv("GFX906_FA_DECODE_V16PPW2");
  const bool v16_two = !(v16p && v16p[0] == '0');
  const char* nt3p = std::getenv("GFX906_FA_DECODE_NT3PPW2");
  const bool nt3_two = !(nt3p && nt3p[0] == '0');
  // 9-16 rows per kv head (two n-tiles, Q^T in registers): two pages per warp
  // in three stages as for one n-tile (config 3 with two query tokens per
  // sequence: 8 kv heads 526 -> 468 us, one kv head 87 -> 77.5 us);
  // GFX906_FA_DECODE_NT2PPW2=0 turns it off (tuning override).
  const char* nt2p = std::getenv("GFX906_FA_DECODE_NT2PPW2");
  const bool nt2_two = !(nt2p && nt2p[0] == '0');
  if (d.tr != NWC_TR && (d.tr ? (d.nt == 1 || (d.nt == 2 && nt2_two)) && vq8t : mt == 1) && 2 * d.P <= (d.HG == 1 ? MAXP : 8) &&
      need(3, 2 * d.P) <= kSmem) {
    d.ppw = 2;
    d.P *= 2;
    d.nst = 3;
  } else if (nt3_two && d.tr == NWC && d.nt == 3 && 2 * d.P <= 8 && need(2, 2 * d.P) <= kSmem) {
    // 17-24 query rows per kv head (4-token speculative verify at GQA 6):
    // two pages per warp in two stages (three do not fit beside the
    // shared-memory Q tiles), twice the independent work per warp in the
    // latency-bound three-n-tile consumer (config 5's verify rows: decode
    // 1.17 -> 1.01 ms, the mixed step 3.79 -> 3.63 ms);
    // GFX906_FA_DECODE_NT3PPW2=0 turns it off (tuning override).
    d.ppw = 2;
    d.P *= 2;
    d.nst = 2;
  } else if (v16_two && d.tr == NWC && v16 && d.nt == 1 && 2 * d.P <= MAXP && need(2, 2 * d.P) <= kSmem) {
    d.ppw = 2;
    d.P *= 2;
    d.nst = need(3, d.P) <= kSmem ? 3 : 2;
  } else {
    d.nst = need(MAXST, d.P) <= kSmem ? MAXST : 3;
    if (need(d.nst, d.P) > kSmem) return cudaErrorInvalidValue;
  }
  d.stage_bytes = d.P * (d.kpage + d.vpage);
  // K pages then V pages, or (joint) K and V of each page adjacent
  d.joint = vq8t && d.kwhole && d.HGN == 1 && p.v_page_stride == p.k_page_stride && p.v_head_stride == d.vrec &&
            p.v_cache == p.k_cache + (int64_t)PAGE * Hkv * d.rb_k;
  if (d.joint) {
    d.kps = d.vps = d.kpage + d.vpage;
    d.vbase = d.kpage;
  } else {
    d.kps = d.kpage;
    d.vps = d.vpage;
    d.vbase = d.P * d.kpage;
  }
  d.q_off = d.nst * d.stage_bytes;
  d.cpre_off = d.q_off;
  d.qtr_off = d.q_off + (((d.nranks + 1) * 4 + 15) & ~15);
  if (d.tr) d.tr_tab = choose_tr_table(d);
  d.scale_log2 = p.scale * kLog2e;
  if (p.softcap > 0.f) {
    d.cap_in = p.scale / p.softcap;
    d.cap_out = p.softcap * kLog2e;
  }
  // chunking: enough chunks to keep every SM busy several times over
  const int sms = num_sms();
  d.nstreams = sms * d.NG;                 // transposed kernels: one CTA per SM
  const int max_pages = (p.max_kv + PAGE - 1) / PAGE;
  const int64_t est_pages = (int64_t)p.num_seqs * d.HGN * max_pages / 2 + 1;   // lengths ~ U[0, max]
  const int64_t want = est_pages / ((int64_t)sms * d.NG * 6);   // items per group stream
  int cp = (int)std::min<int64_t>(std::max<int64_t>(want, 16), 512);
  // at most kCombineMaxParts partials per (sequence, kv head)
  cp = std::max<int>(cp, (int)(((int64_t)max_pages + kCombineMaxParts - 1) / kCombineMaxParts));
  if (const char* e = std::getenv("GFX906_FA_DECODE_CHUNK")) {   // tuning override: pages per chunk
    const int v = std::atoi(e);
    if (v > 0) cp = std::max<int>(v, (int)(((int64_t)max_pages + kCombineMaxParts - 1) / kCombineMaxParts));
  }
  cp = ((cp + d.ppw - 1) / d.ppw) * d.ppw;
  d.CP = cp;
  d.S_max = max_pages == 0 ? 1 : (max_pages + cp - 1) / cp;
  d.n_items = p.num_seqs * d.HGN * d.S_max;
  return cudaSuccess;
}

// Workspace: [0, 256) work-queue counter; rank prefix sums (transposed
// kernels); partial O rows; (max, sum) per partial row.
static size_t decode_ws_rows(const DecodeParams& d) {
  if (d.tr) return ((size_t)d.nstreams + d.nranks) * d.HG * d.R_pad;   // slots s + rank
  return (size_t)d.p.num_seqs * d.p.num_heads_kv * d.S_max * d.R_pad;
}
static size_t decode_ws_cpre(const DecodeParams& d) {
  return d.tr ? (((size_t)d.nranks + 1) * sizeof(int) + 255) & ~(size_t)255 : 0;
}
static size_t decode_ws_bytes(const DecodeParams& d) {
  const size_t rows = decode_ws_rows(d);
  const size_t o = rows * dec::D * sizeof(float);
  return 256 + decode_ws_cpre(d) + ((o + 255) & ~(size_t)255) + rows * sizeof(float2) + 256;
}


}  // namespace g9


using namespace g9;

extern "C" size_t gfx906_fa_decode_workspace_size(const G9AttnBatch* batch) {
  if (!batch) return 0;
  DecodeParams d;
  int mt;
  if (plan_decode(*batch, d, mt) != cudaSuccess) return 0;
  return decode_ws_bytes(d);
}

extern "C" cudaError_t gfx906_fa_decode_splitk(const G9AttnBatch* batch, void* workspace,
                                               size_t workspace_bytes, cudaStream_t stream) {
  if (!batch) return cudaErrorInvalidValue;
  DecodeParams d;
  int mt;
  cudaError_t e = plan_decode(*batch, d, mt);
  if (e != cudaSuccess) return e;
  if (batch->num_seqs == 0 || batch->seq_q == 0) return cudaSuccess;
  if (!workspace || workspace_bytes < decode_ws_bytes(d) || ((uintptr_t)workspace & 15)) return cudaErrorInvalidValue;
  {
    // [0, 256): work-queue counter; then partial O and (max, sum) rows
    const size_t rows = decode_ws_rows(d), cp = decode_ws_cpre(d);
    uint8_t* w = reinterpret_cast<uint8_t*>(workspace);
    d.counter = reinterpret_cast<unsigned int*>(w);
    d.cpre_g = reinterpret_cast<int*>(w + 256);
    d.opart = reinterpret_cast<float*>(w + 256 + cp);
    d.ml = reinterpret_cast<float2*>(w + 256 + cp + (((rows * dec::D * sizeof(float)) + 255) & ~(size_t)255));
    // the queue-driven kernels claim items from the counter; the transposed
    // kernels split statically and never read it
    if (!d.tr) {
      cudaError_t ze = cudaMemsetAsync(d.counter, 0, sizeof(unsigned int), stream);
      if (ze != cudaSuccess) return ze;
    }
  }
  const int vt = batch->v_fmt;
  // general score path: additive mask, soft-cap or sliding window
  const bool mask = batch->mask != nullptr || batch->softcap > 0.f || batch->window > 0;
#define G9_DEC(MT_, VT_, MK_) \
  if (mt == MT_ && vt == VT_ && mask == MK_) return launch_decode_t<MT_, VT_, MK_>(d, stream);
  G9_DEC(1, 0, false) G9_DEC(2, 0, false) G9_DEC(1, 1, false) G9_DEC(2, 1, false)
  G9_DEC(1, 2, false) G9_DEC(2, 2, false) G9_DEC(1, 3, false) G9_DEC(2, 3, false)
  G9_DEC(1, 0, true) G9_DEC(2, 0, true) G9_DEC(1, 1, true) G9_DEC(2, 1, true)
  G9_DEC(1, 2, true) G9_DEC(2, 2, true) G9_DEC(1, 3, true) G9_DEC(2, 3, true)
#undef G9_DEC
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of gfx906_fa_decode_splitk.
//
// Some callers cannot allocate device memory at call time -- code running
// where cudaMalloc is forbidden or unavailable (inside a custom allocator's
// own callbacks, a runtime that owns every byte of the device heap, or a
// plugin host with a fixed memory budget).  For them the split-K partial
// results live in this file-scope device array instead of a caller-provided
// workspace.  It is g_decode_noalloc_scratch below: kNoAllocScratchBytes
// (32 MiB), held by every GPU that loads the library until the process
// exits.  Host code must not use the array's name as a device pointer; the
// device address is looked up once per device with cudaGetSymbolAddress.
// ---------------------------------------------------------------------------
namespace g9 {
constexpr size_t kNoAllocScratchBytes = (size_t)32 << 20;
static __device__ __align__(256) uint8_t g_decode_noalloc_scratch[kNoAllocScratchBytes];
}  // namespace g9

#include <mutex>

// The calling thread's current CUDA context (driver handle, through the
// runtime's driver entry point), or null if it cannot be queried.
static void* current_context() {
  typedef int (*CtxGetCurrentFn)(void**);
  static CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
               ? reinterpret_cast<CtxGetCurrentFn>(f)
               : nullptr;
  }();
  void* ctx = nullptr;
  if (fn) fn(&ctx);
  return ctx;
}

extern "C" cudaError_t gfx906_fa_decode_splitk_noalloc(const G9AttnBatch* batch, cudaStream_t stream) {
  if (!batch) return cudaErrorInvalidValue;
  // size check before anything touches the device
  DecodeParams d;
  int mt;
  cudaError_t e = plan_decode(*batch, d, mt);
  if (e != cudaSuccess) return e;
  const size_t need = decode_ws_bytes(d);
  if (need > kNoAllocScratchBytes) return cudaErrorInvalidValue;   // batch too large for the static scratch
  // per-device address of the scratch array, looked up on the first call on
  // each device (that first call should come before any stream capture).
  // The address belongs to the module instance of the context that is
  // current, so the cache is keyed on that context as well: after a device
  // reset, or from another context on the same device, it is looked up again.
  constexpr int kMaxDevices = 64;
  static void* addr[kMaxDevices] = {};
  static void* addr_ctx[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  void* ctx = current_context();
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev] || addr_ctx[dev] != ctx) {
      void* p = nullptr;
      if ((e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch)) != cudaSuccess) return e;
      addr[dev] = p;
      addr_ctx[dev] = ctx;
    }
    ptr = addr[dev];
  }
  // Nothing in the array has to be cleared by the caller: the work-queue
  // counter at its start is zeroed by the call itself (cudaMemsetAsync on the
  // stream) whenever the chosen kernel reads it, and every partial result the
  // combine step reads is written earlier in the same call.
  return gfx906_fa_decode_splitk(batch, ptr, kNoAllocScratchBytes, stream);
}

