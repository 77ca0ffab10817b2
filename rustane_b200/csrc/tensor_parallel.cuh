// Tensor-parallel forward (the reference's head- and hidden-sharded layer,
// layer.rs:1906-2053,4943-5139; shard outputs summed on the CPU at layer.rs:2018, 5121):
// the exchange of the row-parallel projections' partial sums over NCCL, sequence parallel
// (reduce-scatter + all-gather) or all-reduce, in chunks of sequences that overlap the
// other chunk's GEMMs.
//
// Included by bridge.cu inside its internal namespace, after the context, the GEMM and
// attention launchers and the NCCL loader it uses, and before enqueue_forward, which
// dispatches to these functions for tensor-parallel contexts.
#pragma once

// Tensor-parallel forward in chunks of sequences on two streams: the compute stream
// runs each chunk's QKV, attention and O projection, then (after that chunk's
// all-reduce) its residual + norm, W1/W3 and down projection; the communication
// stream all-reduces each chunk's fp32 partial projection as soon as it is written,
// while the compute stream works on the other chunks. Same math as the one-stream
// path, chunk by chunk (rows are independent outside attention, and attention stays
// within a sequence).
cudaError_t enqueue_forward_tp_chunked(cb_ctx* c, int batch, int chunks, float softcap,
                                       cudaStream_t st) {
  const cb_model_config& cfg = c->cfg;
  const int S = cfg.seq, d = cfg.dim, hid = c->hidden_l, V = cfg.vocab, L = cfg.nlayers;
  const int T = batch * S, bc = batch / chunks, Tc = bc * S;
  const int H = c->heads_l, Hk = c->kv_heads_l, qd = c->q_dim, kvd = c->kv_dim, nq = c->n_qkv;
  const float alpha = 1.0f / sqrtf(2.0f * (float)L);
  cudaStream_t cs = c->comm_stream;
  DeviceInfo dt = device_info(c->device);
  dt.sms = std::max(1, dt.sms - tp_comm_sms(c->tp_world));
  dt.pair_clusters = std::max(1, std::min(dt.pair_clusters, dt.sms / 2));
  cudaError_t e;
#define TRYC(...)                                     \
  do {                                                \
    if ((e = (__VA_ARGS__)) != cudaSuccess) return e; \
  } while (0)
  auto nccl_sum = [&](float* buf, size_t n) -> cudaError_t {
    ncclResult_t nr = nccl_api().all_reduce(buf, buf, n, ncclFloat32, ncclSum, c->comm, cs);
    if (nccl_settle(c, nr, "ncclAllReduce") != ncclSuccess) return cudaErrorUnknown;
    return cudaSuccess;
  };
  cudaEvent_t* ev_proj = c->tp_ev;               // projection of chunk j written
  cudaEvent_t* ev_sum = c->tp_ev + TP_MAX_CHUNKS;  // chunk j's all-reduce done
  const int m_qkv = pick_mode(Tc, nq, dt), m_o = pick_mode(Tc, d, dt);
  const int m_13 = pick_mode(Tc, 2 * hid, dt);

  embed_rmsnorm_kernel<<<(T + ROW_WARPS - 1) / ROW_WARPS, ROW_WARPS * 32, 0, st>>>(
      c->tokens, c->embed, c->gamma, c->x, c->xn, T, d, V, c->dev_err);
  TRYC(cudaGetLastError());
  // the communication stream joins the capture here
  TRYC(cudaEventRecord(c->tp_ev[3 * TP_MAX_CHUNKS], st));
  TRYC(cudaStreamWaitEvent(cs, c->tp_ev[3 * TP_MAX_CHUNKS], 0));
  for (int l = 0; l < L; ++l) {
    // attention half: QKV, attention, O per chunk; O partials all-reduced on cs
    for (int j = 0; j < chunks; ++j) {
      const size_t r0 = (size_t)j * Tc;
      if (l > 0) {  // previous layer's down projection, summed: residual + RMSNorm(gamma1)
        TRYC(cudaStreamWaitEvent(st, ev_sum[j], 0));
        TRYC(launch_add_rmsnorm(c->x + r0 * d, c->x + r0 * d, c->delta32 + r0 * d,
                                c->gamma + (size_t)l * 2 * d, c->xn + r0 * d, Tc, d, st));
      }
      __half* qj = c->q + r0 * qd;
      __half* kj = c->k + r0 * kvd;
      __half* vj = c->v + r0 * kvd;
      CUtensorMap ta, tq, tk, tv, to;
      if (!make_tmap(&ta, c->xn + r0 * d, d, Tc, 1, 128) ||
          !make_tmap(&to, c->attn + r0 * qd, qd, Tc, 1, 128) ||
          !make_tmap_qkv(&tq, qj, (uint64_t)Tc * H, FA_BQ) ||
          !make_tmap_qkv(&tk, kj, (uint64_t)Tc * Hk, FA_BKV) ||
          !make_tmap_qkv(&tv, vj, (uint64_t)Tc * Hk, FA_BKV))
        return cudaErrorInvalidValue;
      {
        EpiQkvRope ep{qj, kj, vj, c->rope, S, H, Hk};
        TRYC(launch_gemm(m_qkv, ta, c->tm_wqkv[0], c->tm_wqkv[1], Tc, nq, d, l, ep, c->dev_err,
                         dt, st));
      }
      TRYC(launch_attention(S % FA_BQ == 0 ? &tq : nullptr, &tk, &tv, qj, kj, vj,
                            c->attn + r0 * qd, bc, H, Hk, S, c->dev_err, st));
      {
        EpiScaledF32 ep{c->delta32 + r0 * d, d, alpha};
        TRYC(launch_gemm(m_o, to, c->tm_wo[0], c->tm_wo[1], Tc, d, qd, l, ep, c->dev_err, dt,
                         st));
      }
      TRYC(cudaEventRecord(ev_proj[j], st));
      TRYC(cudaStreamWaitEvent(cs, ev_proj[j], 0));
      TRYC(nccl_sum(c->delta32 + r0 * d, (size_t)Tc * d));
      TRYC(cudaEventRecord(ev_sum[j], cs));
    }
    // FFN half: residual + RMSNorm(gamma2), W1/W3 + SwiGLU, down; partials all-reduced on cs
    for (int j = 0; j < chunks; ++j) {
      const size_t r0 = (size_t)j * Tc;
      TRYC(cudaStreamWaitEvent(st, ev_sum[j], 0));
      TRYC(launch_add_rmsnorm(c->x + r0 * d, c->x + r0 * d, c->delta32 + r0 * d,
                              c->gamma + (size_t)l * 2 * d + d, c->xn + r0 * d, Tc, d, st));
      CUtensorMap ta, tg;
      if (!make_tmap(&ta, c->xn + r0 * d, d, Tc, 1, 128) ||
          !make_tmap(&tg, c->g + r0 * hid, hid, Tc, 1, 128))
        return cudaErrorInvalidValue;
      {
        EpiSwiglu ep{c->g + r0 * hid, hid};
        TRYC(launch_gemm(m_13, ta, c->tm_w13[0], c->tm_w13[1], Tc, 2 * hid, d, l, ep, c->dev_err,
                         dt, st));
      }
      {
        EpiScaledF32 ep{c->delta32 + r0 * d, d, alpha};
        TRYC(launch_gemm(m_o, tg, c->tm_w2[0], c->tm_w2[1], Tc, d, hid, l, ep, c->dev_err, dt,
                         st));
      }
      TRYC(cudaEventRecord(ev_proj[j], st));
      TRYC(cudaStreamWaitEvent(cs, ev_proj[j], 0));
      TRYC(nccl_sum(c->delta32 + r0 * d, (size_t)Tc * d));
      TRYC(cudaEventRecord(ev_sum[j], cs));
    }
  }
  for (int j = 0; j < chunks; ++j) {  // last residual + final RMSNorm; joins cs back
    const size_t r0 = (size_t)j * Tc;
    TRYC(cudaStreamWaitEvent(st, ev_sum[j], 0));
    TRYC(launch_add_rmsnorm(c->x + r0 * d, c->x + r0 * d, c->delta32 + r0 * d, c->gamma_final,
                            c->xn + r0 * d, Tc, d, st));
  }
  const DeviceInfo& di = device_info(c->device);
  const int m_head = pick_mode(T, V, di);
  const int nparts = (V + mode_block_n(m_head) - 1) / mode_block_n(m_head);
  {
    EpiCrossEntropy ep{};
    ep.part = c->ce_part;
    ep.nparts = nparts;
    ep.targets = c->targets;
    ep.tgt_logit = c->tgt_logit;
    ep.softcap = softcap;
    TRYC(launch_gemm(m_head, c->tm_xn, c->tm_embed[0], c->tm_embed[1], T, V, d, 0, ep,
                     c->dev_err, di, st));
  }
  const int row_blocks = (T + ROW_WARPS - 1) / ROW_WARPS;
  ce_finalize_kernel<<<row_blocks, ROW_WARPS * 32, 0, st>>>(c->ce_part, nparts, c->tgt_logit,
                                                            c->tok_loss, c->block_sums, T);
  TRYC(cudaGetLastError());
  loss_mean_kernel<<<1, 256, 0, st>>>(c->block_sums, row_blocks, T, c->loss);
  TRYC(cudaGetLastError());
#undef TRYC
  return cudaSuccess;
}

// Chunks for the tensor-parallel forward: CB_TP_CHUNKS (1 = one stream), else 2 when
// the batch splits evenly.
int tp_chunks(const cb_ctx* c, int batch) {
  static const int forced = [] {
    const char* e = getenv("CB_TP_CHUNKS");
    return e ? atoi(e) : 0;
  }();
  int n = forced > 0 ? forced : 2;
  n = std::min(n, TP_MAX_CHUNKS);
  while (n > 1 && batch % n != 0) --n;
  return c->tp_world > 1 ? n : 1;
}

// How the tensor-parallel ranks combine the row-parallel projections (O, down), from
// CB_TP_REDUCE (read once per process):
//   "sp16" (default) sequence parallel: each projection's partial sums are written in fp16
//     and reduce-scattered over the token rows, each rank adds the sums of its own rows to
//     the residual and normalises them, and the normalised fp16 rows are all-gathered for
//     the next column-parallel GEMM (2 + 2 bytes per element cross NVLink, against 8 for
//     an fp32 all-reduce, and the residual + RMSNorm runs on 1/world of the rows);
//   "sp32" the same with fp32 partial sums (4 + 2 bytes);
//   "allreduce" the fp32 partial sums are all-reduced and every rank keeps every row.
enum TpReduce { TP_ALLREDUCE = 0, TP_SP16 = 1, TP_SP32 = 2 };
int tp_reduce_mode() {
  static const int mode = [] {
    const char* e = getenv("CB_TP_REDUCE");
    if (e && !strcmp(e, "allreduce")) return (int)TP_ALLREDUCE;
    if (e && !strcmp(e, "sp32")) return (int)TP_SP32;
    return (int)TP_SP16;
  }();
  return mode;
}

// Sequence-parallel tensor-parallel forward: the reference's head / hidden split of the
// layer (layer.rs:1906-2053,4943-5139, shard outputs summed on the CPU at layer.rs:2018,
// 5121) with the sum done as a reduce-scatter over the token rows.
// Rows: the batch's T tokens in `chunks` chunks of Tc rows; within chunk j rank r owns rows
// [j Tc + r Tl, j Tc + (r + 1) Tl), Tl = Tc / world. Per layer and chunk:
//   compute stream: QKV (every row of the chunk, this rank's heads), attention, O
//     projection -> partial alpha * (A Wo) in delta (fp16) or delta32 (fp32);
//   comm stream:    reduce-scatter of the partials (a rank receives the sums of its own
//     rows), residual add + RMSNorm of those rows (x, xn), all-gather of the normalised
//     fp16 rows into every rank's xn; then the same after W1/W3 -> down.
// The compute stream works on the other chunk while one chunk's rows are exchanged (NCCL
// capped at tp_comm_sms(world) CTAs, the GEMMs on the other SMs). A rank keeps the residual x
// only for its own rows; after the last layer the final rows of x are all-gathered too
// (sampled logits read them). The LM head and the loss run over all rows on every rank,
// so every rank returns the same loss and per-token losses.
// With `prof` (eager profiling, chunks == 1) everything runs on `st`, events between
// the launches.
cudaError_t enqueue_forward_tp_sp(cb_ctx* c, int batch, int chunks, float softcap,
                                  cudaStream_t st, bool prof, bool f16) {
  const cb_model_config& cfg = c->cfg;
  const int S = cfg.seq, d = cfg.dim, hid = c->hidden_l, V = cfg.vocab, L = cfg.nlayers;
  const int T = batch * S, bc = batch / chunks, Tc = bc * S, G = c->tp_world, Tl = Tc / G;
  const int rk = c->tp_rank;
  const int H = c->heads_l, Hk = c->kv_heads_l, qd = c->q_dim, kvd = c->kv_dim, nq = c->n_qkv;
  const float alpha = 1.0f / sqrtf(2.0f * (float)L);  // layer.rs:4420
  const bool two = !prof && c->comm_stream != nullptr;
  cudaStream_t cs = two ? c->comm_stream : st;
  DeviceInfo dt = device_info(c->device);
  if (two) {  // the GEMMs leave tp_comm_sms(world) SMs to NCCL
    dt.sms = std::max(1, dt.sms - tp_comm_sms(c->tp_world));
    dt.pair_clusters = std::max(1, std::min(dt.pair_clusters, dt.sms / 2));
  }
  const ncclDataType_t part_type = f16 ? ncclHalf : ncclFloat32;
  const size_t esz = f16 ? 2 : 4;
  char* part = f16 ? reinterpret_cast<char*>(c->delta) : reinterpret_cast<char*>(c->delta32);
  cudaError_t e;
  int ev = 0;
  auto mark = [&](int cls, double flops, double bytes) {
    if (!prof) return;
    c->ev_class.push_back(cls);
    c->ev_flops.push_back(flops);
    c->ev_bytes.push_back(bytes);
    cudaEventRecord(c->events[++ev], st);
  };
  if (prof) {
    c->ev_class.clear();
    c->ev_flops.clear();
    c->ev_bytes.clear();
    cudaEventRecord(c->events[0], st);
  }
#define TRYS(...)                                     \
  do {                                                \
    if ((e = (__VA_ARGS__)) != cudaSuccess) return e; \
  } while (0)
  cudaEvent_t* ev_proj = c->tp_ev;                 // chunk j's partial projection written
  cudaEvent_t* ev_rows = c->tp_ev + TP_MAX_CHUNKS;  // chunk j's normalised rows gathered
  const int m_qkv = pick_mode(Tc, nq, dt), m_o = pick_mode(Tc, d, dt);
  const int m_13 = pick_mode(Tc, 2 * hid, dt);
  const double Tcd = (double)Tc;

  embed_rmsnorm_kernel<<<(T + ROW_WARPS - 1) / ROW_WARPS, ROW_WARPS * 32, 0, st>>>(
      c->tokens, c->embed, c->gamma, c->x, c->xn, T, d, V, c->dev_err);
  TRYS(cudaGetLastError());
  mark(K_EMBED_NORM, 0, (double)T * (4 + d * (2 + 4 + 2)));
  if (two) {  // the communication stream joins the capture here
    TRYS(cudaEventRecord(c->tp_ev[3 * TP_MAX_CHUNKS], st));
    TRYS(cudaStreamWaitEvent(cs, c->tp_ev[3 * TP_MAX_CHUNKS], 0));
  }
  // Chunk j's partials -> sums of this rank's rows -> residual + RMSNorm(gamma) -> every
  // rank's normalised rows (and, after the last layer, the residual rows themselves).
  auto exchange = [&](int j, const float* gamma, bool last) -> cudaError_t {
    const size_t r0 = (size_t)j * Tc, own = r0 + (size_t)rk * Tl;
    if (two) {
      TRYS(cudaEventRecord(ev_proj[j], st));
      TRYS(cudaStreamWaitEvent(cs, ev_proj[j], 0));
    }
    ncclResult_t nr = nccl_api().reduce_scatter(part + r0 * d * esz, part + own * d * esz,
                                                (size_t)Tl * d, part_type, ncclSum, c->comm, cs);
    if (nccl_settle(c, nr, "ncclReduceScatter") != ncclSuccess) return cudaErrorUnknown;
    mark(K_RSCATTER, 0, Tcd * d * esz);
    TRYS(f16 ? launch_add_rmsnorm(c->x + own * d, c->x + own * d, c->delta + own * d, gamma,
                                  c->xn + own * d, Tl, d, cs)
             : launch_add_rmsnorm(c->x + own * d, c->x + own * d, c->delta32 + own * d, gamma,
                                  c->xn + own * d, Tl, d, cs));
    mark(K_RMSNORM, 0, (double)Tl * d * (4 + esz + 4 + 2));
    nr = nccl_api().all_gather(c->xn + own * d, c->xn + r0 * d, (size_t)Tl * d, ncclHalf,
                               c->comm, cs);
    if (nccl_settle(c, nr, "ncclAllGather") != ncclSuccess) return cudaErrorUnknown;
    mark(K_AGATHER, 0, Tcd * d * 2);
    if (last) {
      nr = nccl_api().all_gather(c->x + own * d, c->x + r0 * d, (size_t)Tl * d, ncclFloat32,
                                 c->comm, cs);
      if (nccl_settle(c, nr, "ncclAllGather") != ncclSuccess) return cudaErrorUnknown;
      mark(K_AGATHER, 0, Tcd * d * 4);
    }
    if (two) TRYS(cudaEventRecord(ev_rows[j], cs));
    return cudaSuccess;
  };
  const double attn_flops = 2.0 * 2.0 * (double)bc * H * 128.0 * S * (S + 1) / 2.0;
  for (int l = 0; l < L; ++l) {
    for (int j = 0; j < chunks; ++j) {  // attention half
      const size_t r0 = (size_t)j * Tc;
      if (two && l > 0) TRYS(cudaStreamWaitEvent(st, ev_rows[j], 0));
      __half* qj = c->q + r0 * qd;
      __half* kj = c->k + r0 * kvd;
      __half* vj = c->v + r0 * kvd;
      CUtensorMap ta, tq, tk, tv, to;
      if (!make_tmap(&ta, c->xn + r0 * d, d, Tc, 1, 128) ||
          !make_tmap(&to, c->attn + r0 * qd, qd, Tc, 1, 128) ||
          !make_tmap_qkv(&tq, qj, (uint64_t)Tc * H, FA_BQ) ||
          !make_tmap_qkv(&tk, kj, (uint64_t)Tc * Hk, FA_BKV) ||
          !make_tmap_qkv(&tv, vj, (uint64_t)Tc * Hk, FA_BKV))
        return cudaErrorInvalidValue;
      {
        EpiQkvRope ep{qj, kj, vj, c->rope, S, H, Hk};
        TRYS(launch_gemm(m_qkv, ta, c->tm_wqkv[0], c->tm_wqkv[1], Tc, nq, d, l, ep, c->dev_err,
                         dt, st));
      }
      mark(K_GEMM_QKV, 2.0 * Tcd * nq * d, Tcd * d * 2 + (double)nq * d * 2 + Tcd * nq * 2);
      TRYS(launch_attention(S % FA_BQ == 0 ? &tq : nullptr, &tk, &tv, qj, kj, vj,
                            c->attn + r0 * qd, bc, H, Hk, S, c->dev_err, st));
      mark(K_ATTN, attn_flops, Tcd * (qd + 2 * kvd) * 2 + Tcd * qd * 2);
      if (f16) {
        EpiScaledF16 ep{c->delta + r0 * d, d, alpha};
        TRYS(launch_gemm(m_o, to, c->tm_wo[0], c->tm_wo[1], Tc, d, qd, l, ep, c->dev_err, dt, st));
      } else {
        EpiScaledF32 ep{c->delta32 + r0 * d, d, alpha};
        TRYS(launch_gemm(m_o, to, c->tm_wo[0], c->tm_wo[1], Tc, d, qd, l, ep, c->dev_err, dt, st));
      }
      mark(K_GEMM_O, 2.0 * Tcd * d * qd, Tcd * qd * 2 + (double)d * qd * 2 + Tcd * d * esz);
      TRYS(exchange(j, c->gamma + (size_t)l * 2 * d + d, false));
    }
    const bool last = l + 1 == L;
    const float* g_next = last ? c->gamma_final : c->gamma + (size_t)(l + 1) * 2 * d;
    for (int j = 0; j < chunks; ++j) {  // FFN half
      const size_t r0 = (size_t)j * Tc;
      if (two) TRYS(cudaStreamWaitEvent(st, ev_rows[j], 0));
      CUtensorMap ta, tg;
      if (!make_tmap(&ta, c->xn + r0 * d, d, Tc, 1, 128) ||
          !make_tmap(&tg, c->g + r0 * hid, hid, Tc, 1, 128))
        return cudaErrorInvalidValue;
      {
        EpiSwiglu ep{c->g + r0 * hid, hid};
        TRYS(launch_gemm(m_13, ta, c->tm_w13[0], c->tm_w13[1], Tc, 2 * hid, d, l, ep, c->dev_err,
                         dt, st));
      }
      mark(K_GEMM_W13, 2.0 * Tcd * 2 * hid * d, Tcd * d * 2 + 2.0 * hid * d * 2 + Tcd * hid * 2);
      if (f16) {
        EpiScaledF16 ep{c->delta + r0 * d, d, alpha};
        TRYS(launch_gemm(m_o, tg, c->tm_w2[0], c->tm_w2[1], Tc, d, hid, l, ep, c->dev_err, dt, st));
      } else {
        EpiScaledF32 ep{c->delta32 + r0 * d, d, alpha};
        TRYS(launch_gemm(m_o, tg, c->tm_w2[0], c->tm_w2[1], Tc, d, hid, l, ep, c->dev_err, dt, st));
      }
      mark(K_GEMM_W2, 2.0 * Tcd * d * hid, Tcd * hid * 2 + (double)d * hid * 2 + Tcd * d * esz);
      TRYS(exchange(j, g_next, last));
    }
  }
  if (two)  // join the communication stream back
    for (int j = 0; j < chunks; ++j) TRYS(cudaStreamWaitEvent(st, ev_rows[j], 0));
  const DeviceInfo& di = device_info(c->device);
  const int m_head = pick_mode(T, V, di);
  const int nparts = (V + mode_block_n(m_head) - 1) / mode_block_n(m_head);
  {
    EpiCrossEntropy ep{};
    ep.part = c->ce_part;
    ep.nparts = nparts;
    ep.targets = c->targets;
    ep.tgt_logit = c->tgt_logit;
    ep.softcap = softcap;
    TRYS(launch_gemm(m_head, c->tm_xn, c->tm_embed[0], c->tm_embed[1], T, V, d, 0, ep,
                     c->dev_err, di, st));
  }
  mark(K_GEMM_HEAD, 2.0 * T * (double)V * d,
       (double)T * d * 2 + (double)V * d * 2 + (double)T * nparts * 8 + T * 8.0);
  const int row_blocks = (T + ROW_WARPS - 1) / ROW_WARPS;
  ce_finalize_kernel<<<row_blocks, ROW_WARPS * 32, 0, st>>>(c->ce_part, nparts, c->tgt_logit,
                                                            c->tok_loss, c->block_sums, T);
  TRYS(cudaGetLastError());
  mark(K_CE_FINAL, 0, (double)T * nparts * 8 + T * 8.0);
  loss_mean_kernel<<<1, 256, 0, st>>>(c->block_sums, row_blocks, T, c->loss);
  TRYS(cudaGetLastError());
  mark(K_LOSS_MEAN, 0, row_blocks * 4.0);
#undef TRYS
  return cudaSuccess;
}
