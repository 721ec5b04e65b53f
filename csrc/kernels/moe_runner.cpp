// Native executor of one progressive MoE layer on one rank.
//
// The runner owns no policy: the Python layer (revealaiccl_b200/moe/layer.py)
// allocates every buffer, maps the peers' symmetric regions and hands the
// runner device pointers once.  `forward(delayed)` then enqueues the whole
// layer — router chunks on the router stream, and on the comm stream the
// per-trigger control plane, the revealed-only dispatches (each right after
// its trigger in the early arm, all after the final trigger in the delayed
// arm), the expert plan, both grouped GEMMs, the return rows and signals and
// the combine — with no host synchronisation.  `capture`/`replay` record the
// same sequence once in a CUDA graph and relaunch it (the call's sequence
// number lives in device memory, so replays need no new parameters).
//
// Orchestration being replaced: scripts/run_r4_a0_c0_full_moe.py:264-839
// (_run_arm: producer thread + host consume/schedule/build/communicate loop).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "launchers.h"
#include "moe_kernels.h"
#include "tma_host.h"

namespace {

using raiccl::GemmSegment;

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename T>
T* ptr(const py::dict& t, const char* key) {
  if (!t.contains(key)) throw std::invalid_argument(std::string("missing tensor ") + key);
  py::object o = t[key];
  if (o.is_none()) return nullptr;
  torch::Tensor x = o.cast<torch::Tensor>();
  if (!x.is_cuda()) throw std::invalid_argument(std::string("tensor not on CUDA: ") + key);
  if (!x.is_contiguous()) throw std::invalid_argument(std::string("tensor not contiguous: ") + key);
  return reinterpret_cast<T*>(x.data_ptr());
}

template <typename T>
T* opt_ptr(const py::dict& t, const char* key) {
  if (!t.contains(key)) return nullptr;
  return ptr<T>(t, key);
}

int geti(const py::dict& d, const char* key) {
  if (!d.contains(key)) throw std::invalid_argument(std::string("missing int ") + key);
  return d[key].cast<int>();
}

class MoELayerRunner {
 public:
  MoELayerRunner(py::dict ints, py::dict tensors, std::vector<int64_t> peer_bases,
                 std::vector<int64_t> chunk_offsets, int64_t router_stream, int64_t comm_stream)
      : tensors_(tensors), chunk_offsets_(chunk_offsets.begin(), chunk_offsets.end()) {
    router_ = reinterpret_cast<cudaStream_t>(router_stream);
    comm_ = reinterpret_cast<cudaStream_t>(comm_stream);
    device_ = tensors["tokens"].cast<torch::Tensor>().device().index();
    c10::cuda::CUDAGuard guard(device_);
    if (tensors.contains("trace")) {
      auto tt = tensors["trace"].cast<torch::Tensor>();
      TORCH_CHECK(tt.is_cuda() && tt.is_contiguous() && tt.nbytes() % sizeof(raiccl::TraceSlot) == 0,
                  "trace must be a contiguous CUDA buffer of 32-byte slots");
      trace_ = reinterpret_cast<raiccl::TraceSlot*>(tt.data_ptr());
      trace_cap_ = (int)(tt.nbytes() / sizeof(raiccl::TraceSlot));
    }
    // keep every tensor alive for the runner's lifetime
    for (auto item : tensors) held_.push_back(py::reinterpret_borrow<py::object>(item.second));

    auto& d = dims_;
    d.world = geti(ints, "world");
    d.rank = geti(ints, "rank");
    d.tokens = geti(ints, "tokens");
    d.hidden = geti(ints, "hidden");
    d.out_dim = geti(ints, "out_dim");
    d.experts = geti(ints, "experts");
    d.expert_slots = geti(ints, "expert_slots");
    d.top_k = geti(ints, "top_k");
    d.chunks = geti(ints, "chunks");
    partial_ = geti(ints, "partial_chunks");
    d.n_desc = partial_ < d.chunks ? partial_ + 1 : d.chunks;
    feat_bf16_ = geti(ints, "feat_bf16") != 0;
    out_bf16_ = geti(ints, "out_bf16") != 0;
    d.feat_bytes = feat_bf16_ ? 2 : 4;
    d.out_bytes = out_bf16_ ? 2 : 4;
    d.placement = geti(ints, "placement");
    d.gate_mode = geti(ints, "gate_mode");
    d.mask_mode = geti(ints, "mask_mode");
    d.ctl_per_chunk = geti(ints, "ctl_per_chunk");
    d.ctl_nodes = geti(ints, "ctl_nodes");
    d.pad0 = 0;
    d.cap = d.tokens;
    ffn_ = geti(ints, "ffn");
    n1_ = geti(ints, "n1");
    act1_ = geti(ints, "act1");
    bn1_ = geti(ints, "bn1");
    bn2_ = geti(ints, "bn2");
    {
      // CTA-pair GEMM kernels (256 x BN tiles on clusters of two SMs) for BN >= 64
      pdl_ = !ints.contains("pdl") || geti(ints, "pdl") != 0;
      const bool allow = !ints.contains("gemm_pair") || geti(ints, "gemm_pair") != 0;
      pair1_ = allow && bn1_ >= 64;
      pair2_ = allow && bn2_ >= 64;
      // swapped tail tiles: CTA-pair kernel at BN = 256, not for SwiGLU (its
      // tile interleaves gate and up columns)
      const int swap = ints.contains("gemm_swap_max") ? geti(ints, "gemm_swap_max") : 128;
      if (swap < 0 || swap > 256) throw std::invalid_argument("gemm_swap_max must be in [0, 256]");
      swap1_ = pair1_ && bn1_ == 256 && act1_ != (int)raiccl::Act::kSwiGLU ? swap : 0;
      swap2_ = pair2_ && bn2_ == 256 ? swap : 0;
    }
    timeout_ns_ = (unsigned long long)ints["timeout_ns"].cast<int64_t>();
    // Progressive expert side: GEMM-1 (CTA pairs) takes tiles as descriptors
    // arrive; needs the persistent front end (decided below) and its tensors.
    progressive_req_ = pair1_ && (!ints.contains("progressive") || geti(ints, "progressive") != 0) &&
                       tensors.contains("tile_list") && tensors.contains("tile_word") &&
                       tensors.contains("ticket_counter") && tensors.contains("pair_tickets");
    dispatch_ctas_ = ints.contains("dispatch_ctas") ? geti(ints, "dispatch_ctas") : 0;
    router_ring_ = !ints.contains("router_ring") || geti(ints, "router_ring") != 0;
    dispatch_groups_ = !ints.contains("dispatch_groups") || geti(ints, "dispatch_groups") != 0;
    router_wsmem_ = !ints.contains("router_wsmem") || geti(ints, "router_wsmem") != 0;
    router_tc_ = !ints.contains("router_tc") || geti(ints, "router_tc") != 0;
    gemm_ksplit_ = !ints.contains("gemm_ksplit") || geti(ints, "gemm_ksplit") != 0;
    max_cands_ = geti(ints, "max_cands");
    log_stride_ = geti(ints, "log_stride");
    max_ctl_tokens_ = geti(ints, "max_ctl_tokens");
    grid_sms_ = geti(ints, "sms");
    control_serial_ = ints.contains("control_serial") && geti(ints, "control_serial") != 0;
    if (d.world < 1 || d.world > raiccl::kMaxRanks) throw std::invalid_argument("world size 1..8");
    if ((int)peer_bases.size() != d.world) throw std::invalid_argument("peer base count != world");
    if ((int)chunk_offsets_.size() != d.chunks + 1) throw std::invalid_argument("chunk offsets");
    if (d.top_k > 8 || d.experts > 255) throw std::invalid_argument("top_k <= 8 and experts <= 255");
    if (d.chunks > 60) throw std::invalid_argument("at most 60 chunks");
    layout_ = raiccl::make_sym_layout(d);
    for (int r = 0; r < raiccl::kMaxRanks; ++r) peers_.base[r] = r < d.world ? (unsigned long long)peer_bases[r] : 0ULL;

    // tensor maps of both GEMMs are built once (every buffer is fixed)
    const long long rows = (long long)d.expert_slots * d.world * d.cap;
    const CUtensorMapDataType dt = feat_bf16_ ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const int eb = d.feat_bytes, bk = 128 / eb;
    void* recv_feat = reinterpret_cast<uint8_t*>(peers_.base[d.rank]) + layout_.recv_feat;
    ta1_ = raiccl::make_tmap_2d_sw128(recv_feat, dt, eb, rows, d.hidden, d.hidden, 128, bk);
    tb1_ = raiccl::make_tmap_2d_sw128(ptr<void>(tensors, "w1"), dt, eb, (uint64_t)d.expert_slots * n1_, d.hidden, d.hidden, pair1_ ? bn1_ / 2 : bn1_, bk);
    ta2_ = raiccl::make_tmap_2d_sw128(ptr<void>(tensors, "h"), dt, eb, rows, ffn_, ffn_, 128, bk);
    // 8-row boxes of the same A tensors: swapped tail tiles stage only the rows they use
    ta1n_ = raiccl::make_tmap_2d_sw128(recv_feat, dt, eb, rows, d.hidden, d.hidden, 8, bk);
    ta2n_ = raiccl::make_tmap_2d_sw128(ptr<void>(tensors, "h"), dt, eb, rows, ffn_, ffn_, 8, bk);
    tb2_ = raiccl::make_tmap_2d_sw128(ptr<void>(tensors, "w2"), dt, eb, (uint64_t)d.expert_slots * d.out_dim, ffn_, ffn_, pair2_ ? bn2_ / 2 : bn2_, bk);
    // tensor-core router (bf16): the token matrix in 128-token boxes and the
    // router weights in one box of E rounded up to 16 rows (rows past E read as zero)
    if (feat_bf16_ && router_tc_ && d.hidden % 64 == 0 && d.experts <= 64 && d.top_k <= 8) {
      const uint32_t npad = (uint32_t)std::max(16, (d.experts + 15) / 16 * 16);
      tx_router_ = raiccl::make_tmap_2d_sw128(ptr<void>(tensors, "tokens"), dt, eb, (uint64_t)d.tokens, d.hidden,
                                              d.hidden, 128, bk);
      tw_router_ = raiccl::make_tmap_2d_sw128(ptr<void>(tensors, "router_w"), dt, eb, (uint64_t)d.experts, d.hidden,
                                              d.hidden, npad, bk);
      have_tc_router_ = true;
    }

    {
      int coop = 0;
      cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device_);
      const int mode = ints.contains("frontend") ? geti(ints, "frontend") : 1;
      use_frontend_ = coop != 0 && mode != 0 && tensors.contains("chunk_words") && tensors.contains("disp_base") &&
                      tensors.contains("desc_ready");
      if (tensors.contains("chunk_words")) {
        chunk_words_ = ptr<int>(tensors, "chunk_words");
        // [C] chunk_done, [C, E] chunk_counts, then GEMM-1's split-K tile
        // tickets (whatever the tensor holds beyond), all zeroed per call
        n_chunk_words_ = (int)tensors["chunk_words"].cast<torch::Tensor>().numel();
        const int base = d.chunks * (1 + d.experts);
        if (n_chunk_words_ > base && tensors.contains("ksplit_partial") && !tensors["ksplit_partial"].is_none()) {
          ksplit_partial_ = ptr<float>(tensors, "ksplit_partial");
          ksplit_ticket_ = chunk_words_ + base;
          const long long rows = tensors["ksplit_partial"].cast<torch::Tensor>().numel() / (128LL * bn1_);
          ksplit_entries_ = (int)std::min<long long>(n_chunk_words_ - base, rows);
        }
      }
    }
    ck(cudaEventCreateWithFlags(&ev_start_, cudaEventDisableTiming), "cudaEventCreate");
    ev_chunk_.resize(d.chunks);
    for (auto& e : ev_chunk_) ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    ev_ctl_.resize(d.n_desc);
    for (auto& e : ev_ctl_) ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    ck(cudaEventCreateWithFlags(&ev_disp_done_, cudaEventDisableTiming), "cudaEventCreate");
    ck(cudaEventCreateWithFlags(&ev_plan_, cudaEventDisableTiming), "cudaEventCreate");
    ck(cudaEventCreateWithFlags(&ev_retmeta_, cudaEventDisableTiming), "cudaEventCreate");
    ck(cudaEventCreateWithFlags(&ev_call_done_, cudaEventDisableTiming), "cudaEventCreate");
    ck(cudaEventCreateWithFlags(&ev_entry_, cudaEventDisableTiming), "cudaEventCreate");
    ev_tok_.resize(d.chunks);
    for (auto& e : ev_tok_) ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    ck(cudaStreamCreateWithFlags(&sig_, cudaStreamNonBlocking), "cudaStreamCreate");
    if (tensors.contains("tok_ready")) {
      tok_ready_ = ptr<unsigned long long>(tensors, "tok_ready");
      tok_ready_all_ = tok_ready_ + d.chunks;
      stream_pending_ = tok_ready_ + d.chunks + 1;
    }
    // dispatch chain: its own stream, so trigger q+1's control overlaps dispatch q
    ck(cudaStreamCreateWithFlags(&disp_, cudaStreamNonBlocking), "cudaStreamCreate");
  }

  ~MoELayerRunner() {
    for (int a = 0; a < 2; ++a) {
      if (exec_[a]) cudaGraphExecDestroy(exec_[a]);
      if (graph_[a]) cudaGraphDestroy(graph_[a]);
    }
    for (auto& e : ev_chunk_) cudaEventDestroy(e);
    for (auto& e : ev_ctl_) cudaEventDestroy(e);
    if (ev_disp_done_) cudaEventDestroy(ev_disp_done_);
    if (ev_plan_) cudaEventDestroy(ev_plan_);
    if (ev_retmeta_) cudaEventDestroy(ev_retmeta_);
    if (ev_call_done_) cudaEventDestroy(ev_call_done_);
    if (ev_entry_) cudaEventDestroy(ev_entry_);
    for (auto& e : ev_tok_) cudaEventDestroy(e);
    if (sig_) cudaStreamDestroy(sig_);
    if (ev_start_) cudaEventDestroy(ev_start_);
    if (disp_) cudaStreamDestroy(disp_);
  }

  // Enqueue one layer call; returns the number of kernels launched.
  int forward(bool delayed) {
    c10::cuda::CUDAGuard guard(device_);
    const auto& d = dims_;
    const py::dict& t = tensors_;
    int launches = 0;
    auto* status = ptr<raiccl::DeviceStatus>(t, "status");
    auto* epoch = ptr<unsigned long long>(t, "epoch");
    auto* sent_base = ptr<int>(t, "sent_base");
    auto* desc_counts = ptr<int>(t, "desc_counts");
    auto* done_counter = ptr<int>(t, "done_counter");
    auto* permit = ptr<unsigned long long>(t, "permit");
    auto* expert_ids = ptr<int>(t, "expert_ids");
    auto* gates = ptr<float>(t, "gates");
    auto* chunk_offsets_dev = ptr<int>(t, "chunk_offsets");

    trace_labels_.clear();
    raiccl::TraceSlot* reset_slot = trace_slot("layer_reset", -1);
    const bool progressive = progressive_req_ && use_frontend_;
    raiccl::launch_layer_reset(sent_base, d.experts, desc_counts, d.n_desc, done_counter, epoch, trace_,
                               trace_cap_, chunk_words_, n_chunk_words_, tok_ready_all_, stream_pending_, comm_,
                               progressive ? ptr<unsigned int>(t, "ticket_counter") : nullptr);
    (void)reset_slot;
    ++launches;

    // router chunks
    raiccl::RouterParams rp{};
    rp.tokens = ptr<void>(t, "tokens");
    rp.weight = ptr<void>(t, "router_w");
    rp.bias = ptr<float>(t, "router_b");
    rp.block_mask = opt_ptr<uint8_t>(t, "block_mask");
    const float* chunk_bias = opt_ptr<float>(t, "chunk_bias");
    rp.hidden = d.hidden;
    rp.experts = d.experts;
    rp.top_k = d.top_k;
    rp.gate_mode = d.gate_mode;
    rp.mask_mode = d.mask_mode;
    rp.expert_ids = expert_ids;
    rp.gates = gates;
    auto launch_routers = [&]() {
      ck(cudaEventRecord(ev_start_, comm_), "cudaEventRecord");
      ck(cudaStreamWaitEvent(router_, ev_start_, 0), "cudaStreamWaitEvent");
      for (int c = 0; c < d.chunks; ++c) {
        rp.row0 = (int)chunk_offsets_[c];
        rp.row1 = (int)chunk_offsets_[c + 1];
        rp.chunk_bias = chunk_bias ? chunk_bias + (long long)c * d.experts : nullptr;
        if (rp.row1 > rp.row0) {
          rp.trace = trace_slot("router", c);
          raiccl::launch_router(rp, feat_bf16_, router_);
          ++launches;
        }
        ck(cudaEventRecord(ev_chunk_[c], router_), "cudaEventRecord");
      }
    };

    // control plane + dispatch
    raiccl::ControlParams cp{};
    cp.plan.E = geti_t("plan_E");
    cp.plan.G = geti_t("plan_G");
    cp.n_group_members = geti_t("plan_NGM");
    cp.n_edge_group_members = geti_t("plan_NEGM");
    cp.n_tmpl = geti_t("plan_NT");
    cp.max_tmpl = geti_t("plan_MT");
    cp.force_serial = control_serial_ ? 1 : 0;
    cp.plan.V = d.ctl_nodes;
    cp.st.max_tokens = max_ctl_tokens_;
    cp.max_cands = max_cands_;
    cp.chunks = d.chunks;
    {
      // plan, state, scalars and scratch live in one blob (control_layout.h)
      const auto L = raiccl::control_layout(raiccl::ControlDims{
          cp.plan.E, cp.plan.G, cp.plan.V, cp.st.max_tokens, cp.n_group_members, cp.n_edge_group_members,
          cp.n_tmpl, cp.max_cands, d.chunks});
      auto blob_t = t["ctl_blob"].cast<torch::Tensor>();
      TORCH_CHECK(blob_t.is_cuda() && blob_t.is_contiguous() && blob_t.nbytes() >= (size_t)L.total,
                  "ctl_blob must be a contiguous CUDA buffer of control_layout total bytes");
      cp.blob = reinterpret_cast<uint8_t*>(blob_t.data_ptr());
      auto at = [&](int a) { return cp.blob + L.off[a]; };
      cp.plan.edge_src = reinterpret_cast<int32_t*>(at(raiccl::kCtlEdgeSrc));
      cp.plan.edge_tgt = reinterpret_cast<int32_t*>(at(raiccl::kCtlEdgeTgt));
      cp.plan.cap_units = reinterpret_cast<int64_t*>(at(raiccl::kCtlCap));
      cp.plan.group_limits = reinterpret_cast<int64_t*>(at(raiccl::kCtlGroupLimits));
      cp.plan.group_ptr = reinterpret_cast<int32_t*>(at(raiccl::kCtlGroupPtr));
      cp.plan.group_members = reinterpret_cast<int32_t*>(at(raiccl::kCtlGroupMembers));
      cp.plan.edge_group_ptr = reinterpret_cast<int32_t*>(at(raiccl::kCtlEdgeGroupPtr));
      cp.plan.edge_group_members = reinterpret_cast<int32_t*>(at(raiccl::kCtlEdgeGroupMembers));
      cp.plan.distances = reinterpret_cast<int32_t*>(at(raiccl::kCtlDistances));
      cp.plan.tmpl_ptr = reinterpret_cast<int32_t*>(at(raiccl::kCtlTmplPtr));
      cp.plan.tmpl_edge = reinterpret_cast<int32_t*>(at(raiccl::kCtlTmplEdge));
      cp.plan.tmpl_src = reinterpret_cast<int32_t*>(at(raiccl::kCtlTmplSrc));
      cp.plan.tmpl_tgt = reinterpret_cast<int32_t*>(at(raiccl::kCtlTmplTgt));
      cp.plan.tmpl_tdist = reinterpret_cast<int32_t*>(at(raiccl::kCtlTmplTdist));
      cp.st.sources = reinterpret_cast<int32_t*>(at(raiccl::kCtlSources));
      cp.st.destinations = reinterpret_cast<int32_t*>(at(raiccl::kCtlDestinations));
      cp.st.holders = at(raiccl::kCtlHolders);
      cp.st.ready = at(raiccl::kCtlReady);
      cp.st.committed = at(raiccl::kCtlCommitted);
      cp.st.residual = at(raiccl::kCtlResidual);
      cp.st.remaining_hops = reinterpret_cast<int32_t*>(at(raiccl::kCtlRemainingHops));
      cp.st.residual_demand = reinterpret_cast<int64_t*>(at(raiccl::kCtlResidualDemand));
      cp.st.link_credits = reinterpret_cast<int64_t*>(at(raiccl::kCtlLinkCredits));
      cp.st.group_credits = reinterpret_cast<int64_t*>(at(raiccl::kCtlGroupCredits));
      cp.st.scratch_selected = at(raiccl::kCtlScratchSelected);
      cp.st.scratch_seen = at(raiccl::kCtlScratchSeen);
      cp.st.scratch_edge_load = reinterpret_cast<int64_t*>(at(raiccl::kCtlScratchEdgeLoad));
      cp.scalars = reinterpret_cast<long long*>(at(raiccl::kCtlScalars));
      cp.cand_buf = reinterpret_cast<raiccl::sched::Cand*>(at(raiccl::kCtlCands));
      cp.keep_buf = reinterpret_cast<int*>(at(raiccl::kCtlKeep));
      cp.action_buf = reinterpret_cast<int64_t*>(at(raiccl::kCtlActions));
    }
    cp.expert_ids = expert_ids;
    cp.chunk_offsets = chunk_offsets_dev;
    cp.top_k = d.top_k;
    cp.chunks = d.chunks;
    cp.partial_chunks = partial_;
    cp.ctl_per_chunk = d.ctl_per_chunk;
    cp.ctl_nodes = d.ctl_nodes;
    cp.log_stride = log_stride_;
    cp.log = ptr<int>(t, "ctl_log");
    cp.permit = permit;
    cp.epoch = epoch;
    cp.status = status;

    raiccl::DispatchParams dp{};
    dp.dims = d;
    dp.layout = layout_;
    dp.peers = peers_;
    dp.tokens = rp.tokens;
    dp.expert_ids = expert_ids;
    dp.gates = gates;
    dp.token_ids = ptr<long long>(t, "token_ids");
    dp.feat_digest = ptr<long long>(t, "feat_digest");
    dp.checksum_base = ptr<long long>(t, "checksum_base");
    dp.chunk_offsets = chunk_offsets_dev;
    dp.sent_base = sent_base;
    dp.desc_counts = desc_counts;
    dp.done_counter = done_counter;
    dp.permit = permit;
    dp.epoch = epoch;
    dp.status = status;
    dp.peer_counters = opt_ptr<unsigned long long>(t, "peer_counters");

    auto dispatch = [&](int q) {
      const int c_lo = q < partial_ ? q : partial_;
      const int c_hi = q < partial_ ? q : d.chunks - 1;
      dp.desc = q;
      dp.t0 = (int)chunk_offsets_[c_lo];
      dp.t1 = (int)chunk_offsets_[c_hi + 1];
      const int ntok = dp.t1 - dp.t0;
      const int tpc = std::max(1, 16 / d.top_k);
      const int grid = std::max(1, std::min(4 * grid_sms_, (ntok + tpc - 1) / tpc));
      dp.trace = trace_slot("dispatch", q);
      dp.fault_skip_signal = (q == fault_skip_signal_desc_) ? 1 : 0;
      raiccl::launch_dispatch(dp, feat_bf16_, grid, disp_);
      ++launches;
    };
    bool front = use_frontend_;
    if (front) {
      // router + control plane + dispatch: one persistent cooperative launch
      raiccl::FrontendParams fp{};
      fp.rp = rp;
      fp.rp.chunk_bias = chunk_bias;
      fp.cp = cp;
      fp.dp = dp;
      fp.chunk_done = chunk_words_;
      fp.chunk_counts = chunk_words_ + d.chunks;
      fp.disp_base = ptr<int>(t, "disp_base");
      fp.desc_ready = ptr<unsigned long long>(t, "desc_ready");
      fp.delayed = delayed ? 1 : 0;
      fp.fault_skip_desc = fault_skip_signal_desc_;
      fp.timeout_ns = timeout_ns_;
      fp.cta_clock = opt_ptr<unsigned long long>(t, "fe_clock");
      // streamed calls: the workers wait for each chunk and digest the rows they route
      fp.digest_out = ptr<long long>(t, "feat_digest");
      fp.csbase_out = ptr<long long>(t, "checksum_base");
      fp.tok_ready = tok_ready_;
      fp.tok_ready_all = tok_ready_all_;
      fp.early_dependents = progressive ? 1 : 0;
      fp.dispatch_ctas = progressive ? dispatch_ctas_ : 0;
      fp.ring_slots = router_ring_ ? 1 : 0;  // a request: launch_frontend sizes the ring
      fp.dispatch_groups = dispatch_groups_ ? 1 : 0;
      fp.w_off = router_wsmem_ ? 1 : 0;  // a request: launch_frontend places the weights
      if (have_tc_router_) {  // a request: launch_frontend sizes the stages
        fp.tc_router = 1;
        fp.tmap_x = tx_router_;
        fp.tmap_w = tw_router_;
      }
      const size_t mark = trace_labels_.size();
      fp.trace = trace_slot("frontend", -1);
      raiccl::TraceSlot* first = nullptr;
      for (int c = 0; c < d.chunks; ++c) {
        raiccl::TraceSlot* sl = trace_slot("router", c);
        if (c == 0) first = sl;
      }
      for (int q = 0; q < d.n_desc; ++q) trace_slot("control", q);
      for (int q = 0; q < d.n_desc; ++q) trace_slot("dispatch", q);
      fp.phase_trace = (first != nullptr && trace_labels_.size() == mark + 1 + d.chunks + 2 * d.n_desc) ? first
                                                                                                       : nullptr;
      int tcu = 0;
      const bool launched = raiccl::launch_frontend(fp, feat_bf16_, grid_sms_, comm_, &tcu);
      tc_used_ = launched ? tcu : 0;
      if (launched) {
        ++launches;
      } else {
        trace_labels_.resize(mark);
        use_frontend_ = front = false;  // not co-schedulable here: step pipeline from now on
        if (progressive) throw std::runtime_error("progressive expert side needs the persistent front end; "
                                                  "rebuild the layer with progressive=0");
      }
    }
    if (!front) launch_routers();
    // control triggers on comm_ (each after its router chunk); dispatch q on
    // disp_ after control q (early arm) or after the last control (delayed arm)
    for (int q = 0; q < d.n_desc && !front; ++q) {
      const int last_chunk = q < partial_ ? q : d.chunks - 1;
      ck(cudaStreamWaitEvent(comm_, ev_chunk_[last_chunk], 0), "cudaStreamWaitEvent");
      cp.desc = q;
      cp.trace = trace_slot("control", q);
      raiccl::launch_control(cp, comm_);
      ++launches;
      ck(cudaEventRecord(ev_ctl_[q], comm_), "cudaEventRecord");
      if (!delayed) {
        ck(cudaStreamWaitEvent(disp_, ev_ctl_[q], 0), "cudaStreamWaitEvent");
        dispatch(q);
      }
    }
    if (delayed && !front) {
      ck(cudaStreamWaitEvent(disp_, ev_ctl_[d.n_desc - 1], 0), "cudaStreamWaitEvent");
      for (int q = 0; q < d.n_desc; ++q) dispatch(q);
    }
    if (!front) {
      ck(cudaEventRecord(ev_disp_done_, disp_), "cudaEventRecord");
      ck(cudaStreamWaitEvent(comm_, ev_disp_done_, 0), "cudaStreamWaitEvent");
    }

    // expert side
    auto* segs = ptr<GemmSegment>(t, "segs");
    raiccl::PlanParams pp{};
    pp.dims = d;
    pp.layout = layout_;
    pp.peers = peers_;
    pp.segs = segs;
    pp.rows_out = ptr<int>(t, "rows_out");
    pp.epoch = epoch;
    pp.timeout_ns = timeout_ns_;
    pp.status = status;
    pp.trace = trace_slot("expert_plan", -1);
    // the plan also writes both GEMMs' tile tables
    const int S = d.expert_slots * d.world;
    int* prefix1 = ptr<int>(t, "prefix1");
    int* prefix2 = ptr<int>(t, "prefix2");
    pp.prefix1 = prefix1;
    pp.prefix2 = prefix2;
    pp.nblocks1 = n1_ / bn1_;
    pp.nblocks2 = d.out_dim / bn2_;
    pp.bm1 = pair1_ ? 256 : 128;
    pp.bm2 = pair2_ ? 256 : 128;
    int* tail1 = swap1_ ? ptr<int>(t, "tail1") : nullptr;
    int* tail2 = swap2_ ? ptr<int>(t, "tail2") : nullptr;
    pp.tail1 = tail1;
    pp.tail2 = tail2;
    pp.peer_counters = dp.peer_counters;
    pp.swap1 = swap1_;
    pp.swap2 = swap2_;
    if (progressive) {
      auto tl = t["tile_list"].cast<torch::Tensor>();
      pp.tile_list = reinterpret_cast<int32_t*>(tl.data_ptr());
      pp.max_tiles1 = (int)(tl.numel() / 4);
      pp.tile_word = ptr<unsigned long long>(t, "tile_word");
      raiccl::launch_expert_plan_progressive(pp, comm_);
    } else {
      raiccl::launch_expert_plan(pp, comm_, pdl_);
    }
    ++launches;

    auto launch_return_meta_side = [&]() {
    // Return metadata depends only on the plan: it runs on the dispatch
    // stream beside the GEMMs; whichever of it and the combine reports last
    // publishes the return signal.  (A progressive GEMM-1 is launched right
    // behind its planner, so that nothing stands between the two launches.)
    ck(cudaEventRecord(ev_plan_, comm_), "cudaEventRecord");
    ck(cudaStreamWaitEvent(disp_, ev_plan_, 0), "cudaStreamWaitEvent");
    raiccl::ReturnMetaParams rm{};
    rm.dims = d;
    rm.layout = layout_;
    rm.peers = peers_;
    rm.segs = segs;
    rm.status = status;
    rm.trace = trace_slot("return_meta", -1);
    auto* ret_sync = reinterpret_cast<unsigned long long*>(ptr<int64_t>(t, "ret_sync"));
    rm.epoch = epoch;
    rm.ret_sync = ret_sync;
    raiccl::launch_return_meta(rm, grid_sms_, disp_);
    ck(cudaEventRecord(ev_retmeta_, disp_), "cudaEventRecord");
    ++launches;
    };
    auto* ret_sync = reinterpret_cast<unsigned long long*>(ptr<int64_t>(t, "ret_sync"));
    if (!progressive) launch_return_meta_side();

    raiccl::GroupedGemmParams g1{};
    g1.segs = segs;
    g1.tile_prefix = prefix1;
    g1.tail_prefix = tail1;
    g1.swap_max = swap1_;
    g1.num_segs = S;
    g1.N = n1_;
    g1.K = d.hidden;
    g1.bias = opt_ptr<float>(t, "b1");
    g1.row_map = nullptr;
    g1.row_scale = nullptr;
    g1.out_ptrs = reinterpret_cast<void* const*>(ptr<int64_t>(t, "out_ptrs1"));
    g1.ldo = ffn_;
    g1.status = status;
    g1.timeout_ns = timeout_ns_;
    g1.pair = pair1_ ? 1 : 0;
    g1.pdl = pdl_ ? 1 : 0;
    g1.trace = trace_slot("gemm1", -1);
    if (!pair1_ && gemm_ksplit_ && ksplit_partial_ != nullptr) {  // few tiles, long K: split K over idle SMs
      g1.ksplit_partial = ksplit_partial_;
      g1.ksplit_ticket = ksplit_ticket_;
      g1.ksplit_entries = ksplit_entries_;
      g1.ksplit_max = 8;
    }
    if (progressive) {
      g1.progressive = 1;
      g1.pdl = 1;
      g1.tile_list = ptr<int32_t>(t, "tile_list");
      g1.tile_word = ptr<unsigned long long>(t, "tile_word");
      g1.ticket_counter = ptr<unsigned int>(t, "ticket_counter");
      g1.pair_tickets = ptr<unsigned long long>(t, "pair_tickets");
      g1.epoch = epoch;
      if (t["pair_tickets"].cast<torch::Tensor>().numel() < (int64_t)(grid_sms_ / 2) * raiccl::kPairTicketRing * 2)
        throw std::invalid_argument("pair_tickets holds fewer than (sms / 2) * kPairTicketRing * 2 words");
    }
    raiccl::launch_grouped_gemm(!feat_bf16_, feat_bf16_, act1_, bn1_, ta1_, tb1_, g1, grid_sms_, comm_, &ta1n_);
    ++launches;
    if (progressive) launch_return_meta_side();

    raiccl::GroupedGemmParams g2{};
    g2.segs = segs;
    g2.tile_prefix = prefix2;
    g2.tail_prefix = tail2;
    g2.swap_max = swap2_;
    g2.num_segs = S;
    g2.N = d.out_dim;
    g2.K = ffn_;
    g2.bias = opt_ptr<float>(t, "b2");
    g2.row_map = reinterpret_cast<const int*>(reinterpret_cast<uint8_t*>(peers_.base[d.rank]) + layout_.recv_retrow);
    g2.row_scale = reinterpret_cast<const float*>(reinterpret_cast<uint8_t*>(peers_.base[d.rank]) + layout_.recv_gate);
    g2.out_ptrs = reinterpret_cast<void* const*>(ptr<int64_t>(t, "out_ptrs2"));
    g2.ldo = d.out_dim;
    g2.status = status;
    g2.timeout_ns = timeout_ns_;
    g2.pair = pair2_ ? 1 : 0;
    g2.pdl = pdl_ ? 1 : 0;
    g2.trace = trace_slot("gemm2_return", -1);
    raiccl::launch_grouped_gemm(!feat_bf16_, out_bf16_, 0, bn2_, ta2_, tb2_, g2, grid_sms_, comm_, &ta2n_);
    ++launches;

    raiccl::CombineParams cb{};
    cb.dims = d;
    cb.layout = layout_;
    cb.peers = peers_;
    cb.out = ptr<void>(t, "out");
    cb.epoch = epoch;
    cb.timeout_ns = timeout_ns_;
    cb.status = status;
    cb.trace = trace_slot("combine", -1);
    cb.ret_sync = ret_sync;
    raiccl::launch_combine(cb, out_bf16_, grid_sms_, comm_, pdl_);
    ++launches;
    // join the dispatch stream (the metadata grid finished long before)
    ck(cudaStreamWaitEvent(comm_, ev_retmeta_, 0), "cudaStreamWaitEvent");
    ck(cudaGetLastError(), "MoE layer launch");
    if (!capturing()) call_done();
    return launches;
  }

  // Every executed call (eager or replayed) advances the device epoch by one;
  // the host mirror names the epoch of the next call for streamed inputs.
  bool capturing() const {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    ck(cudaStreamIsCapturing(comm_, &st), "cudaStreamIsCapturing");
    return st != cudaStreamCaptureStatusNone;
  }
  void call_done() {
    ++calls_;
    ck(cudaEventRecord(ev_call_done_, comm_), "cudaEventRecord");
  }

  // One layer call whose token batch is streamed from pinned host memory:
  // chunk c's rows are copied on `copy_stream` and published by a
  // stream-ordered write of this call's epoch into tok_ready[c], which the
  // front end's workers wait for before routing the chunk (so the copy of
  // later chunks overlaps the routing, control and dispatch of earlier ones).
  // The copies start once everything already enqueued on the comm stream has
  // run (the previous call, which reads the token buffer, and any work the
  // caller put there, such as the start event of a timed region), so a call's
  // host-to-device traffic lies inside any window that the caller opens on
  // the comm stream before the call.
  int stream_call(int64_t host_ptr, int64_t copy_stream, bool delayed) {
    c10::cuda::CUDAGuard guard(device_);
    if (!use_frontend_ || tok_ready_ == nullptr)
      throw std::runtime_error("streamed inputs need the persistent front end");
    auto* copy = reinterpret_cast<cudaStream_t>(copy_stream);
    const auto& d = dims_;
    const unsigned long long e_next = calls_ + 1;
    const size_t row_bytes = (size_t)d.hidden * d.feat_bytes;
    auto* dst = ptr<uint8_t>(tensors_, "tokens");
    const auto* src = reinterpret_cast<const uint8_t*>(host_ptr);
    ck(write_value(comm_, stream_pending_, 1), "stream write (pending)");
    ck(cudaEventRecord(ev_entry_, comm_), "cudaEventRecord");
    ck(cudaStreamWaitEvent(copy, ev_entry_, 0), "cudaStreamWaitEvent");
    // The copies run back to back on the copy stream; a second stream turns
    // each copy's completion event into its arrival word, so no stream write
    // sits between two copies (each would hold the next copy until it ran).
    ck(cudaStreamWaitEvent(sig_, ev_entry_, 0), "cudaStreamWaitEvent");
    for (int c = 0; c < d.chunks; ++c) {
      const size_t off = (size_t)chunk_offsets_[c] * row_bytes;
      const size_t n = (size_t)(chunk_offsets_[c + 1] - chunk_offsets_[c]) * row_bytes;
      if (n) ck(cudaMemcpyAsync(dst + off, src + off, n, cudaMemcpyHostToDevice, copy), "cudaMemcpyAsync");
      ck(cudaEventRecord(ev_tok_[c], copy), "cudaEventRecord");
      ck(cudaStreamWaitEvent(sig_, ev_tok_[c], 0), "cudaStreamWaitEvent");
      ck(write_value(sig_, tok_ready_ + c, e_next), "stream write (chunk)");
    }
    // the caller's streams see the copies through the copy stream
    ck(cudaStreamWaitEvent(copy, ev_tok_[d.chunks - 1], 0), "cudaStreamWaitEvent");
    const int a = delayed ? 1 : 0;
    if (exec_[a]) {
      ck(cudaGraphLaunch(exec_[a], comm_), "cudaGraphLaunch");
      call_done();
      return graph_launches_[a];
    }
    return forward(delayed);
  }

  // cuStreamWriteValue64 through the runtime's driver entry point: a word
  // written by the stream's front end in stream order, no kernel (a kernel
  // could not start while the cooperative front end holds every SM).
  static cudaError_t write_value(cudaStream_t s, unsigned long long* addr, unsigned long long v) {
    static PFN_cuStreamWriteValue64_v11070 fn = nullptr;
    if (fn == nullptr) {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuStreamWriteValue64", &p, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || p == nullptr)
        return cudaErrorNotSupported;
      fn = reinterpret_cast<PFN_cuStreamWriteValue64_v11070>(p);
    }
    return fn((CUstream)s, (CUdeviceptr)addr, (cuuint64_t)v, CU_STREAM_WRITE_VALUE_DEFAULT) == CUDA_SUCCESS
               ? cudaSuccess
               : cudaErrorUnknown;
  }

  // Record one layer call of the given arm into that arm's CUDA graph slot.
  int capture(bool delayed) {
    c10::cuda::CUDAGuard guard(device_);
    const int a = delayed ? 1 : 0;
    if (exec_[a]) { cudaGraphExecDestroy(exec_[a]); exec_[a] = nullptr; }
    if (graph_[a]) { cudaGraphDestroy(graph_[a]); graph_[a] = nullptr; }
    ck(cudaStreamBeginCapture(comm_, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    int n = 0;
    try {
      n = forward(delayed);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(comm_, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    ck(cudaStreamEndCapture(comm_, &graph_[a]), "cudaStreamEndCapture");
    ck(cudaGraphInstantiate(&exec_[a], graph_[a], 0), "cudaGraphInstantiate");
    graph_launches_[a] = n;
    return n;
  }

  bool has_graph(bool delayed) const { return exec_[delayed ? 1 : 0] != nullptr; }

  int replay(bool delayed) {
    c10::cuda::CUDAGuard guard(device_);
    const int a = delayed ? 1 : 0;
    if (!exec_[a]) throw std::runtime_error("no captured graph for this arm");
    ck(cudaGraphLaunch(exec_[a], comm_), "cudaGraphLaunch");
    call_done();
    return graph_launches_[a];
  }

  // Align all ranks on the device (no host round-trip) before a timed call.
  void device_barrier() {
    c10::cuda::CUDAGuard guard(device_);
    raiccl::BarrierParams bp{};
    bp.dims = dims_;
    bp.layout = layout_;
    bp.peers = peers_;
    bp.counter = ptr<unsigned long long>(tensors_, "bar_counter");
    bp.timeout_ns = timeout_ns_;
    bp.status = ptr<raiccl::DeviceStatus>(tensors_, "status");
    raiccl::launch_device_barrier(bp, comm_);
    ck(cudaGetLastError(), "device barrier launch");
  }

  long long sym_bytes() const { return layout_.total; }
  unsigned long long calls() const { return calls_; }

  // Fault injection for failure-detection tests: the dispatch of descriptor
  // `desc` moves its rows but publishes no ready flag, so every receiver's
  // bounded wait runs out and reports through the status record (-1: off).
  // Takes effect at the next forward() / capture().
  void inject_skip_signal(int desc) { fault_skip_signal_desc_ = desc; }
  bool persistent_frontend() const { return use_frontend_; }
  // the last front-end launch routed on the tensor cores
  bool router_tc_used() const { return use_frontend_ && tc_used_ != 0; }
  bool progressive() const { return progressive_req_ && use_frontend_; }

  py::list trace_labels() const {
    py::list out;
    for (const auto& kv : trace_labels_) out.append(py::make_tuple(kv.first, kv.second));
    return out;
  }

  py::dict layout() const {
    py::dict o;
    o["recv_feat"] = layout_.recv_feat;
    o["recv_meta"] = layout_.recv_meta;
    o["recv_retrow"] = layout_.recv_retrow;
    o["recv_gate"] = layout_.recv_gate;
    o["recv_count"] = layout_.recv_count;
    o["recv_flag"] = layout_.recv_flag;
    o["ret_out"] = layout_.ret_out;
    o["ret_meta"] = layout_.ret_meta;
    o["ret_flag"] = layout_.ret_flag;
    o["bar_flag"] = layout_.bar_flag;
    o["total"] = layout_.total;
    return o;
  }

 private:
  int geti_t(const char* key) const {
    py::object o = tensors_[key];
    return o.cast<int>();
  }

  py::dict tensors_;
  std::vector<py::object> held_;
  std::vector<long long> chunk_offsets_;
  raiccl::MoEDims dims_{};
  raiccl::SymLayout layout_{};
  raiccl::PeerBases peers_{};
  int partial_ = 0, ffn_ = 0, n1_ = 0, act1_ = 0, bn1_ = 0, bn2_ = 0;
  bool pair1_ = false, pair2_ = false;  // GEMM 1 / 2 on the CTA-pair kernel
  int swap1_ = 0, swap2_ = 0;            // GEMM 1 / 2 swapped-tail row limit (0: off)
  bool progressive_req_ = false;         // progressive GEMM-1 requested and possible with the pair kernel
  int dispatch_ctas_ = 0;                // front-end workers that dispatch in progressive mode (0: all)
  bool router_ring_ = true;              // resident batches: token groups stream into shared memory by bulk copies
  bool dispatch_groups_ = true;          // one worker group per descriptor (dispatched side by side)
  bool router_wsmem_ = true;             // router weights copied into each worker's shared memory
  bool router_tc_ = true;                // bf16 batches: tensor-core router units of 128 tokens
  bool gemm_ksplit_ = true;              // one-CTA GEMM-1: split K when the tiles are few
  bool have_tc_router_ = false;          // router tensor maps built (bf16, D % 64 == 0, E <= 64)
  int tc_used_ = 0;                      // the last front-end launch routed on the tensor cores
  CUtensorMap tx_router_{}, tw_router_{};
  bool pdl_ = true;  // plan, GEMMs and combine as programmatic dependents of their predecessors
  int max_cands_ = 0, log_stride_ = 0, max_ctl_tokens_ = 0, grid_sms_ = 148;
  bool control_serial_ = false;  // run the CTA control kernel even where the single-warp one fits
  bool feat_bf16_ = false, out_bf16_ = false;
  unsigned long long timeout_ns_ = 0;
  CUtensorMap ta1_{}, tb1_{}, ta2_{}, tb2_{}, ta1n_{}, ta2n_{};
  cudaStream_t router_ = nullptr, comm_ = nullptr;
  cudaStream_t disp_ = nullptr;
  int device_ = 0;
  int fault_skip_signal_desc_ = -1;
  bool use_frontend_ = false;      // persistent cooperative front end (else one launch per step)
  int* chunk_words_ = nullptr;     // [C] chunk_done + [C * E] chunk_counts, zeroed per call
  float* ksplit_partial_ = nullptr;  // GEMM-1 split-K partial tiles [entries, 128, bn1], or nullptr
  int* ksplit_ticket_ = nullptr;     // GEMM-1 split-K tile tickets (inside chunk_words)
  int ksplit_entries_ = 0;
  int n_chunk_words_ = 0;  // host-side fault injection: descriptor whose ready flags are withheld
  // device trace ring (optional tensor "trace"): one slot per launch of a call
  raiccl::TraceSlot* trace_ = nullptr;
  int trace_cap_ = 0;
  std::vector<std::pair<std::string, int>> trace_labels_;
  raiccl::TraceSlot* trace_slot(const char* kind, int arg) {
    if (trace_ == nullptr || (int)trace_labels_.size() >= trace_cap_) return nullptr;
    trace_labels_.emplace_back(kind, arg);
    return trace_ + (trace_labels_.size() - 1);
  }
  cudaEvent_t ev_start_ = nullptr, ev_disp_done_ = nullptr, ev_plan_ = nullptr, ev_retmeta_ = nullptr;
  cudaEvent_t ev_call_done_ = nullptr;  // end of the last executed call on the comm stream
  cudaEvent_t ev_entry_ = nullptr;      // comm stream at the entry of a streamed call
  std::vector<cudaEvent_t> ev_tok_;     // streamed chunk c copied
  cudaStream_t sig_ = nullptr;          // publishes streamed-chunk arrival words
  unsigned long long calls_ = 0;        // executed calls (== the device epoch after them)
  unsigned long long* tok_ready_ = nullptr;       // [C] streamed-chunk arrival words
  unsigned long long* tok_ready_all_ = nullptr;   // resident-batch word
  unsigned long long* stream_pending_ = nullptr;  // the next reset leaves arrival to the copy stream
  std::vector<cudaEvent_t> ev_chunk_, ev_ctl_;
  cudaGraph_t graph_[2] = {nullptr, nullptr};
  cudaGraphExec_t exec_[2] = {nullptr, nullptr};
  int graph_launches_[2] = {0, 0};
};

// Standalone router launch (tests and the router-only benchmark).
void router_topk(torch::Tensor tokens, torch::Tensor weight, torch::Tensor bias,
                 c10::optional<torch::Tensor> chunk_bias, c10::optional<torch::Tensor> block_mask,
                 int64_t row0, int64_t row1, int64_t top_k, int64_t gate_mode, int64_t mask_mode,
                 torch::Tensor expert_ids, torch::Tensor gates) {
  TORCH_CHECK(tokens.is_cuda() && tokens.is_contiguous() && weight.is_contiguous(), "router: layout");
  TORCH_CHECK(tokens.scalar_type() == weight.scalar_type(), "router: dtypes");
  TORCH_CHECK(tokens.size(1) % (16 / tokens.element_size()) == 0, "router: hidden alignment");
  TORCH_CHECK(weight.size(0) <= 64 && top_k <= 8 && top_k <= weight.size(0), "router: E <= 64, k <= 8");
  TORCH_CHECK(bias.scalar_type() == torch::kFloat32 && expert_ids.scalar_type() == torch::kInt32 &&
                  gates.scalar_type() == torch::kFloat32, "router: aux dtypes");
  c10::cuda::CUDAGuard guard(tokens.device());
  raiccl::RouterParams p{};
  p.tokens = tokens.data_ptr();
  p.weight = weight.data_ptr();
  p.bias = bias.data_ptr<float>();
  p.chunk_bias = chunk_bias ? chunk_bias->data_ptr<float>() : nullptr;
  p.block_mask = block_mask ? block_mask->data_ptr<uint8_t>() : nullptr;
  p.row0 = (int)row0;
  p.row1 = (int)row1;
  p.hidden = (int)tokens.size(1);
  p.experts = (int)weight.size(0);
  p.top_k = (int)top_k;
  p.gate_mode = (int)gate_mode;
  p.mask_mode = (int)mask_mode;
  p.expert_ids = expert_ids.data_ptr<int>();
  p.gates = gates.data_ptr<float>();
  raiccl::launch_router(p, tokens.scalar_type() == torch::kBFloat16, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void feature_digest(torch::Tensor rows, torch::Tensor digest) {
  TORCH_CHECK(rows.is_cuda() && rows.is_contiguous() && rows.dim() == 2, "digest: rows");
  TORCH_CHECK((rows.size(1) * rows.element_size()) % 4 == 0, "digest: row bytes % 4");
  c10::cuda::CUDAGuard guard(rows.device());
  raiccl::launch_feature_digest(rows.data_ptr(), rows.size(1) * rows.element_size(), (int)rows.size(0),
                                reinterpret_cast<long long*>(digest.data_ptr<int64_t>()), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void checksum_base(torch::Tensor token_ids, torch::Tensor digest, torch::Tensor chunk_offsets,
                   int64_t rank, torch::Tensor out) {
  c10::cuda::CUDAGuard guard(token_ids.device());
  raiccl::launch_checksum_base(reinterpret_cast<const long long*>(token_ids.data_ptr<int64_t>()),
                               reinterpret_cast<const long long*>(digest.data_ptr<int64_t>()),
                               chunk_offsets.data_ptr<int>(), (int)chunk_offsets.numel() - 1, (int)rank,
                               (int)token_ids.numel(), reinterpret_cast<long long*>(out.data_ptr<int64_t>()),
                               at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t sym_layout_bytes(py::dict ints) {
  raiccl::MoEDims d{};
  d.world = geti(ints, "world");
  d.tokens = geti(ints, "tokens");
  d.hidden = geti(ints, "hidden");
  d.out_dim = geti(ints, "out_dim");
  d.expert_slots = geti(ints, "expert_slots");
  d.top_k = geti(ints, "top_k");
  d.n_desc = geti(ints, "n_desc");
  d.feat_bytes = geti(ints, "feat_bf16") ? 2 : 4;
  d.out_bytes = geti(ints, "out_bf16") ? 2 : 4;
  d.cap = d.tokens;
  return raiccl::make_sym_layout(d).total;
}

py::dict sym_layout(py::dict ints) {
  raiccl::MoEDims d{};
  d.world = geti(ints, "world");
  d.tokens = geti(ints, "tokens");
  d.hidden = geti(ints, "hidden");
  d.out_dim = geti(ints, "out_dim");
  d.expert_slots = geti(ints, "expert_slots");
  d.top_k = geti(ints, "top_k");
  d.n_desc = geti(ints, "n_desc");
  d.feat_bytes = geti(ints, "feat_bf16") ? 2 : 4;
  d.out_bytes = geti(ints, "out_bf16") ? 2 : 4;
  d.cap = d.tokens;
  auto L = raiccl::make_sym_layout(d);
  py::dict o;
  o["recv_feat"] = L.recv_feat; o["recv_meta"] = L.recv_meta; o["recv_retrow"] = L.recv_retrow;
  o["recv_gate"] = L.recv_gate; o["recv_count"] = L.recv_count; o["recv_flag"] = L.recv_flag;
  o["ret_out"] = L.ret_out; o["ret_meta"] = L.ret_meta; o["ret_flag"] = L.ret_flag;
  o["bar_flag"] = L.bar_flag; o["total"] = L.total;
  py::list guards;
  for (int i = 0; i < raiccl::kSymArrays; ++i) guards.append(L.guard[i]);
  o["guards"] = guards;
  o["guard_bytes"] = raiccl::kGuardBytes;
  return o;
}

py::dict control_layout_py(py::dict dims) {
  const auto L = raiccl::control_layout(raiccl::ControlDims{
      geti(dims, "E"), geti(dims, "G"), geti(dims, "V"), geti(dims, "T"), geti(dims, "n_gm"), geti(dims, "n_egm"),
      geti(dims, "n_tmpl"), geti(dims, "max_cands"), geti(dims, "chunks")});
  static const char* names[raiccl::kCtlArrays] = {
      "edge_src", "edge_tgt", "cap_units", "group_limits", "group_ptr", "group_members", "edge_group_ptr",
      "edge_group_members", "distances", "tmpl_ptr", "tmpl_edge", "tmpl_src", "tmpl_tgt", "tmpl_tdist",
      "st_sources", "st_destinations", "st_holders", "st_ready", "st_committed", "st_residual",
      "st_remaining_hops", "st_residual_demand", "st_link_credits", "st_group_credits", "st_scratch_selected",
      "st_scratch_seen", "st_scratch_edge_load", "ctl_scalars", "ctl_cands", "ctl_keep", "ctl_actions"};
  py::dict arrays;
  for (int i = 0; i < raiccl::kCtlArrays; ++i)
    arrays[names[i]] = py::make_tuple(L.off[i], L.count[i], L.elem[i]);
  py::dict o;
  o["arrays"] = arrays;
  o["state_begin"] = L.state_begin;
  o["state_end"] = L.state_end;
  o["total"] = L.total;
  return o;
}

// Publish `value` at a host-mapped 64-bit word (device pointer) from the
// current stream after `delay_ns` of device time.
void signal_host_flag(int64_t device_ptr, int64_t value, int64_t delay_ns) {
  TORCH_CHECK(device_ptr != 0 && (device_ptr & 7) == 0, "signal_host_flag: 8-byte aligned device pointer");
  TORCH_CHECK(delay_ns >= 0, "signal_host_flag: delay_ns >= 0");
  raiccl::launch_host_flag_signal(reinterpret_cast<unsigned long long*>(device_ptr), (unsigned long long)value,
                                  (unsigned long long)delay_ns, at::cuda::getCurrentCUDAStream());
  ck(cudaGetLastError(), "signal_host_flag");
}

}  // namespace

void register_moe(py::module_& m) {
  py::class_<MoELayerRunner>(m, "MoELayerRunner")
      .def(py::init<py::dict, py::dict, std::vector<int64_t>, std::vector<int64_t>, int64_t, int64_t>(),
           py::arg("ints"), py::arg("tensors"), py::arg("peer_bases"), py::arg("chunk_offsets"),
           py::arg("router_stream"), py::arg("comm_stream"))
      .def("forward", &MoELayerRunner::forward, py::arg("delayed"))
      .def("capture", &MoELayerRunner::capture, py::arg("delayed"))
      .def("replay", &MoELayerRunner::replay, py::arg("delayed"))
      .def("stream_call", &MoELayerRunner::stream_call, py::arg("host_ptr"), py::arg("copy_stream"),
           py::arg("delayed"))
      .def("calls", &MoELayerRunner::calls)
      .def("has_graph", &MoELayerRunner::has_graph, py::arg("delayed"))
      .def("device_barrier", &MoELayerRunner::device_barrier)
      .def("sym_bytes", &MoELayerRunner::sym_bytes)
      .def("trace_labels", &MoELayerRunner::trace_labels)
      .def("inject_skip_signal", &MoELayerRunner::inject_skip_signal, py::arg("desc"))
      .def("persistent_frontend", &MoELayerRunner::persistent_frontend)
      .def("router_tc_used", &MoELayerRunner::router_tc_used)
      .def("progressive", &MoELayerRunner::progressive)
      .def("layout", &MoELayerRunner::layout);
  m.def("router_topk", &router_topk, py::arg("tokens"), py::arg("weight"), py::arg("bias"),
        py::arg("chunk_bias"), py::arg("block_mask"), py::arg("row0"), py::arg("row1"), py::arg("top_k"),
        py::arg("gate_mode"), py::arg("mask_mode"), py::arg("expert_ids"), py::arg("gates"));
  m.def("feature_digest", &feature_digest, py::arg("rows"), py::arg("digest"));
  m.def("checksum_base", &checksum_base, py::arg("token_ids"), py::arg("digest"), py::arg("chunk_offsets"),
        py::arg("rank"), py::arg("out"));
  m.def("sym_layout_bytes", &sym_layout_bytes, py::arg("ints"));
  m.def("sym_layout", &sym_layout, py::arg("ints"));
  m.def("control_layout", &control_layout_py, py::arg("dims"));
  m.def("signal_host_flag", &signal_host_flag, py::arg("device_ptr"), py::arg("value"), py::arg("delay_ns") = 0);
}
