// batch_host.cuh — host side of the batched frame loop (included into
// engine.cu after the Engine definition; kernels in batch_engine.cuh).
#pragma once

namespace qtts {

struct TiledLayer {
    uint8_t * qkv = nullptr, * o = nullptr, * gu = nullptr, * down = nullptr;
};

struct BatchEngine {
    Engine * E = nullptr;
    int dev = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    int Bmax = 0, B = 0, n_max = 0, max_frames = 0, max_pages = 0, n_pages = 0, trail_cap = 0;
    int H = 0, NH = 0, NKV = 0, QD = 0, KD = 0, QKVD = 0, FF = 0, CFF = 0, V0 = 0, V1 = 0, NCB = 0;
    std::vector<TiledLayer> TL, TCP;
    std::vector<uint8_t *> cp_head_t;
    uint8_t * codec_head_t = nullptr;
    std::vector<void *> owned;
    float * x = nullptr, * xcp = nullptr, * qkv = nullptr, * att = nullptr, * hbuf = nullptr;
    float * logits = nullptr, * cp_logits = nullptr, * hidden = nullptr, * trail = nullptr, * pad = nullptr;
    uint8_t * xt = nullptr, * xt2 = nullptr;   // tiled activations: pack target / producer-written
    DevState * st = nullptr;
    SampleParams * sp = nullptr;
    int * codes = nullptr, * page_table = nullptr, * d_err = nullptr;
    __half * pool = nullptr, * cpk = nullptr, * cpv = nullptr;
    float2 * rope_t = nullptr;
    size_t cp_stride = 0, cp_layer = 0;
    cudaGraphExec_t graph = nullptr;
    int graph_B = -1;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float frames_ms = 0.0f;
    int seq_frames = 0;
    std::vector<int> produced;
    int launches = 0;
    // eager per-class profile (events around every launch; not used in the graph)
    enum { BC_PACK = 0, BC_GEMM_QKV, BC_GEMM_O, BC_GEMM_GU, BC_GEMM_DOWN, BC_GEMM_HEAD, BC_ATTN_CP, BC_ATTN_TALKER,
           BC_SAMPLE, BC_OTHER, BC_N };
    bool prof = false;
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> prof_ev;
    int prof_cls = BC_OTHER;
    cudaEvent_t prof_a = nullptr;
    void pb(int cls) {
        if (!prof) return;
        prof_cls = cls;
        cudaEventCreate(&prof_a);
        cudaEventRecord(prof_a, stream);
    }
    void pe() {
        if (!prof) return;
        cudaEvent_t b;
        cudaEventCreate(&b);
        cudaEventRecord(b, stream);
        prof_ev.push_back({prof_cls, {prof_a, b}});
    }

    template <class T>
    bool alloc(T ** p, size_t bytes) {
        if (cudaMalloc(p, bytes) != cudaSuccess) { err = "batch: out of device memory"; return false; }
        owned.push_back(*p);
        return true;
    }

    ~BatchEngine() {
        cudaSetDevice(dev);
        if (graph) cudaGraphExecDestroy(graph);
        for (void * p : owned) cudaFree(p);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        if (stream) cudaStreamDestroy(stream);
    }

    bool tile(const DMat & W, const DMat * W2, uint8_t ** out) {
        const int rows_w = W2 ? 2 * W.rows : W.rows;
        if (W.type != W_F16) { err = "batched path: F16 weights only"; return false; }
        if (rows_w % TC_BM || W.cols % TC_BK || (W2 && W.rows % (TC_BM / 2))) { err = "batched path: matrix shape"; return false; }
        if (!alloc(out, (size_t) rows_w * W.cols * 2)) return false;
        k_tile_weights<<<rows_w, 128, 0, stream>>>((const __half *) W.w, W2 ? (const __half *) W2->w : nullptr, rows_w,
                                                  W.cols, *out);
        return cudaGetLastError() == cudaSuccess;
    }

    bool create(Engine * eng, int bmax, int nmax, int mframes) {
        E = eng;
        dev = eng->dev;
        const qtts_config & c = eng->cfg;
        if (bmax < 1 || bmax > 64) { err = "max_batch must be in [1, 64]"; return false; }
        if (c.code_pred_layers <= 0 || c.n_attention_heads % c.n_key_value_heads) { err = "model layout"; return false; }
        Bmax = bmax; n_max = nmax; max_frames = mframes;
        H = c.hidden_size; NH = c.n_attention_heads; NKV = c.n_key_value_heads;
        QD = NH * QTTS_HD; KD = NKV * QTTS_HD; QKVD = QD + 2 * KD;
        FF = c.intermediate_size; CFF = c.code_pred_intermediate_size;
        V0 = c.codec_vocab_size; V1 = c.code_pred_vocab_size; NCB = c.n_codebooks;
        if (V0 > SAMPLE_THREADS * SAMPLE_PER_T || V1 > SAMPLE_THREADS * SAMPLE_PER_T) { err = "vocabulary too large"; return false; }
        if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess) { err = "stream"; return false; }
        cudaEventCreate(&ev0);
        cudaEventCreate(&ev1);
        TL.resize(E->L.size());
        TCP.resize(E->CPL.size());
        auto tl = [&](std::vector<LayerW> & Ls, std::vector<TiledLayer> & T) {
            for (size_t i = 0; i < Ls.size(); ++i)
                if (!tile(Ls[i].qkv, nullptr, &T[i].qkv) || !tile(Ls[i].o, nullptr, &T[i].o) ||
                    !tile(Ls[i].gate, &Ls[i].up, &T[i].gu) || !tile(Ls[i].down, nullptr, &T[i].down))
                    return false;
            return true;
        };
        if (!tl(E->L, TL) || !tl(E->CPL, TCP)) return false;
        cp_head_t.resize(E->cp_head.size());
        for (size_t g = 0; g < E->cp_head.size(); ++g)
            if (!tile(E->cp_head[g], nullptr, &cp_head_t[g])) return false;
        if (!tile(E->codec_head, nullptr, &codec_head_t)) return false;
        const int R = 2 * Bmax;
        const int maxc = std::max(std::max(H, QD), std::max(FF, CFF));
        if (!alloc(&x, sizeof(float) * Bmax * H) || !alloc(&xcp, sizeof(float) * R * H) ||
            !alloc(&qkv, sizeof(float) * R * QKVD) || !alloc(&att, sizeof(float) * R * QD) ||
            !alloc(&hbuf, sizeof(float) * R * std::max(FF, CFF)) || !alloc(&logits, sizeof(float) * Bmax * V0) ||
            !alloc(&cp_logits, sizeof(float) * Bmax * V1) || !alloc(&hidden, sizeof(float) * Bmax * H) ||
            !alloc(&pad, sizeof(float) * H) || !alloc(&xt, (size_t) TC_MAX_N * maxc * 2) ||
            !alloc(&xt2, (size_t) TC_MAX_N * maxc * 2) ||
            !alloc(&st, sizeof(DevState) * Bmax) || !alloc(&sp, sizeof(SampleParams)) ||
            !alloc(&codes, sizeof(int) * Bmax * max_frames * NCB) || !alloc(&d_err, sizeof(int)))
            return false;
        trail_cap = 1024;
        if (!alloc(&trail, sizeof(float) * Bmax * trail_cap * H)) return false;
        max_pages = (n_max + BP_PAGE - 1) / BP_PAGE;
        n_pages = Bmax * max_pages;
        if (!alloc(&pool, sizeof(__half) * bp_page_elems((int) E->L.size(), NKV) * n_pages) ||
            !alloc(&page_table, sizeof(int) * Bmax * max_pages))
            return false;
        std::vector<int> pt((size_t) Bmax * max_pages);
        for (size_t i = 0; i < pt.size(); ++i) pt[i] = (int) i;   // static partition of the pool
        if (cudaMemcpy(page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
            err = "page table"; return false;
        }
        cp_layer = (size_t) 16 * NKV * QTTS_HD;
        cp_stride = cp_layer * E->CPL.size();
        if (!alloc(&cpk, sizeof(__half) * cp_stride * Bmax) || !alloc(&cpv, sizeof(__half) * cp_stride * Bmax)) return false;
        std::vector<float2> rt;
        E->build_rope(rt, n_max, c.rope_theta);
        if (!alloc(&rope_t, sizeof(float2) * rt.size())) return false;
        if (cudaMemcpy(rope_t, rt.data(), sizeof(float2) * rt.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
            err = "rope"; return false;
        }
        const size_t tcs = 201 * 1024;
        if (cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) tcs) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
            cudaFuncSetAttribute(k_attn_paged, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int) paged_attn_smem(n_max, NH / NKV)) != cudaSuccess) {
            err = "kernel attributes (context too long?)"; return false;
        }
        if (paged_attn_smem(n_max, NH / NKV) > 220 * 1024) { err = "max_positions too large for the paged attention"; return false; }
        if (cudaStreamSynchronize(stream) != cudaSuccess || cudaGetLastError() != cudaSuccess) { err = "weight tiling"; return false; }
        return true;
    }

    // Y = W a (+ epilogue) for m activation rows: pack (RMSNorm, F16 / hi-lo) + tcgen05 GEMM.
    // xin == nullptr: the activation tiles are already in xt2 (written by the producer).
    // xt_next: SwiGLU only, also write h as hi/lo tiles into xt2 for the down GEMM.
    void gemm(const uint8_t * wt, int rows_w, int cols, const float * xin, int ldx, int m, const float * norm, int act,
              int epi, float * y, int ldy, const float * resid, float * xn_out = nullptr, bool xt_next = false) {
        const int mp = (m + 15) / 16 * 16;
        const int np = act == TC_ACT_SPLIT ? 2 * mp : mp;
        const uint8_t * xsrc = xt2;
        if (xin) {
            PackArgs pa{};
            pa.x = xin; pa.ldx = ldx; pa.m_real = m; pa.np = np; pa.cols = cols; pa.gain = norm;
            pa.eps = E->cfg.rms_norm_eps; pa.act = act; pa.out = xt; pa.xn_out = xn_out; pa.ldxn = H;
            pb(BC_PACK);
            pdl_launch(k_pack_act, dim3(act == TC_ACT_SPLIT ? np / 2 : np), dim3(256), 0, stream, pa);
            pe();
            launches += 1;
            xsrc = xt;
        }
        GemmTcArgs g{};
        g.w = wt; g.x = xsrc; g.rows_w = rows_w; g.cols = cols; g.np = np; g.m_real = m;
        g.split = act == TC_ACT_SPLIT; g.epi = epi; g.y = y; g.ldy = ldy; g.resid = resid; g.ldr = ldy; g.err = d_err;
        if (xt_next) { g.xt_out = xt2; g.xt_np = 2 * mp; }
        g.ksplit = tc_choose_split(g);
        pb(gemm_cls);
        tc_launch(g, stream);
        pe();
        launches += 1;
    }
    int gemm_cls = BC_GEMM_QKV;

    void cp_layers(int M, bool f32, int pos_static) {
        const int rows = B * M;
        for (size_t il = 0; il < E->CPL.size(); ++il) {
            const LayerW & l = E->CPL[il];
            const TiledLayer & t = TCP[il];
            gemm_cls = BC_GEMM_QKV;
            gemm(t.qkv, QKVD, H, xcp, H, rows, l.attn_norm, TC_ACT_F16, TC_EPI_STORE, qkv, QKVD, nullptr);
            FusedAttn fa{};
            fa.qkv = qkv; fa.ldq = QKVD; fa.n_heads = NH; fa.n_kv_heads = NKV; fa.q_norm = l.q_norm;
            fa.k_norm = l.k_norm; fa.eps = E->cfg.rms_norm_eps; fa.rope = E->rope_cp;
            fa.kc = cpk + il * cp_layer; fa.vc = cpv + il * cp_layer; fa.pos_static = pos_static; fa.M = M;
            fa.f32_mode = f32 ? 1 : 0; fa.scale = 1.0f / sqrtf((float) QTTS_HD); fa.out = att; fa.ldo = QD;
            fa.xt = xt2; fa.xt_np = (rows + 15) / 16 * 16;
            pb(BC_ATTN_CP);
            pdl_launch(k_cp_attn_warp, dim3((B * NH * M + CPW_WARPS - 1) / CPW_WARPS), dim3(CPW_WARPS * 32), 0, stream, fa,
                       cp_stride, (const DevState *) st, B);
            pe();
            gemm_cls = BC_GEMM_O;
            gemm(t.o, H, QD, nullptr, QD, rows, nullptr, TC_ACT_F16, TC_EPI_RESID, xcp, H, xcp);
            gemm_cls = BC_GEMM_GU;
            gemm(t.gu, 2 * CFF, H, xcp, H, rows, l.ffn_norm, TC_ACT_F16, TC_EPI_SWIGLU, hbuf, CFF, nullptr, nullptr, true);
            gemm_cls = BC_GEMM_DOWN;
            gemm(t.down, H, CFF, nullptr, CFF, rows, nullptr, TC_ACT_SPLIT, TC_EPI_RESID, xcp, H, xcp);
            launches += 1;
        }
    }

    void talker_layers() {
        const int G = NH / NKV;
        for (size_t il = 0; il < E->L.size(); ++il) {
            const LayerW & l = E->L[il];
            const TiledLayer & t = TL[il];
            gemm_cls = BC_GEMM_QKV;
            gemm(t.qkv, QKVD, H, x, H, B, l.attn_norm, TC_ACT_F16, TC_EPI_STORE, qkv, QKVD, nullptr);
            PagedAttnArgs pa{};
            pa.qkv = qkv; pa.ldq = QKVD; pa.n_heads = NH; pa.n_kv_heads = NKV; pa.n_layers = (int) E->L.size();
            pa.layer = (int) il; pa.q_norm = l.q_norm; pa.k_norm = l.k_norm; pa.eps = E->cfg.rms_norm_eps;
            pa.rope = rope_t; pa.pool = pool; pa.page_table = page_table; pa.max_pages = max_pages; pa.st = st;
            pa.scale = 1.0f / sqrtf((float) QTTS_HD); pa.out = att; pa.ldo = QD; pa.n_max = n_max;
            pa.xt = xt2; pa.xt_np = (B + 15) / 16 * 16;
            pb(BC_ATTN_TALKER);
            pdl_launch(k_attn_paged, dim3(B * NKV), dim3(PA_THREADS), paged_attn_smem(n_max, G), stream, pa);
            pe();
            gemm_cls = BC_GEMM_O;
            gemm(t.o, H, QD, nullptr, QD, B, nullptr, TC_ACT_F16, TC_EPI_RESID, x, H, x);
            gemm_cls = BC_GEMM_GU;
            gemm(t.gu, 2 * FF, H, x, H, B, l.ffn_norm, TC_ACT_F16, TC_EPI_SWIGLU, hbuf, FF, nullptr, nullptr, true);
            gemm_cls = BC_GEMM_DOWN;
            gemm(t.down, H, FF, nullptr, FF, B, nullptr, TC_ACT_SPLIT, TC_EPI_RESID, x, H, x);
            launches += 1;
        }
    }

    void enqueue_frame() {
        const int NG = NCB - 1;
        launches = 0;
        pb(BC_SAMPLE);
        pdl_launch(k_sample_batch, dim3(B), dim3(SAMPLE_THREADS), 0, stream, (const float *) logits, V0, V0, 0, st,
                   (const SampleParams *) sp, codes, max_frames);
        pe();
        BatchInputArgs ia{};
        ia.H = H; ia.n_cb = NCB; ia.codec_embd = E->codec_embd; ia.cp_embd = E->d_cp_embd; ia.hidden = hidden;
        ia.trailing = trail; ia.trail_cap = trail_cap; ia.pad = pad; ia.st = st;
        ia.mode = IN_CP_PREFILL; ia.out = xcp;
        pdl_launch(k_inputs_batch, dim3(B), dim3(256), 0, stream, ia);
        cp_layers(2, true, 0);
        gemm_cls = BC_GEMM_HEAD;
        gemm(cp_head_t[0], V1, H, xcp + H, 2 * H, B, E->cp_out_norm, TC_ACT_F16, TC_EPI_STORE, cp_logits, V1, nullptr);
        pb(BC_SAMPLE);
        pdl_launch(k_sample_batch, dim3(B), dim3(SAMPLE_THREADS), 0, stream, (const float *) cp_logits, V1, V1, 1, st,
                   (const SampleParams *) sp, codes, max_frames);
        pe();
        for (int gs = 1; gs < NG; ++gs) {
            ia.mode = IN_CP_STEP; ia.g = gs;
            pdl_launch(k_inputs_batch, dim3(B), dim3(256), 0, stream, ia);
            cp_layers(1, false, gs + 1);
            gemm_cls = BC_GEMM_HEAD;
            gemm(cp_head_t[gs], V1, H, xcp, H, B, E->cp_out_norm, TC_ACT_F16, TC_EPI_STORE, cp_logits, V1, nullptr);
            pb(BC_SAMPLE);
            pdl_launch(k_sample_batch, dim3(B), dim3(SAMPLE_THREADS), 0, stream, (const float *) cp_logits, V1, V1, gs + 1,
                       st, (const SampleParams *) sp, codes, max_frames);
            pe();
            launches += 2;
        }
        ia.mode = IN_TALKER; ia.out = x;
        pdl_launch(k_inputs_batch, dim3(B), dim3(256), 0, stream, ia);
        talker_layers();
        gemm_cls = BC_GEMM_HEAD;
        gemm(codec_head_t, V0, H, x, H, B, E->out_norm, TC_ACT_F16, TC_EPI_STORE, logits, V0, nullptr, hidden);
        pdl_launch(k_frame_end_batch, dim3((B + 127) / 128), dim3(128), 0, stream, st, B);
        launches += 5;
    }

    bool capture() {
        if (graph) { cudaGraphExecDestroy(graph); graph = nullptr; }
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) { err = "capture"; return false; }
        enqueue_frame();
        if (cudaStreamEndCapture(stream, &g) != cudaSuccess) { err = "capture end"; return false; }
        const cudaError_t e = cudaGraphInstantiate(&graph, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) { err = std::string("graph instantiate: ") + cudaGetErrorString(e); return false; }
        graph_B = B;
        return true;
    }

    int begin(int n, const qtts_generate_params * ps) {
        if (n < 1 || n > Bmax) { err = "batch size out of range"; return -1; }
        const qtts_config & c = E->cfg;
        std::vector<DevState> hs(n);
        for (int b = 0; b < n; ++b) {
            if (ps[b].max_len > max_frames) { err = "max_len exceeds the batch's max_frames"; return -1; }
            if (E->begin(&ps[b]) < 0) { err = "prefill of sequence " + std::to_string(b) + ": " + E->err; return -1; }
            const int plen = E->sess.prefill_len, tlen = E->sess.trailing_len;
            if (plen + ps[b].max_len + 1 > n_max) { err = "prompt + max_len exceeds max_positions"; return -1; }
            if (tlen > trail_cap) { err = "too many trailing text rows"; return -1; }
            dim3 grid(plen, (unsigned) E->L.size());
            k_kv_to_pages<<<grid, 256, 0, E->stream>>>(E->kc, E->vc, E->n_ctx, plen, (int) E->L.size(), NKV,
                                                       page_table + (size_t) b * max_pages, pool);
            cudaMemcpyAsync(logits + (size_t) b * V0, E->logits, sizeof(float) * V0, cudaMemcpyDeviceToDevice, E->stream);
            cudaMemcpyAsync(hidden + (size_t) b * H, E->hidden, sizeof(float) * H, cudaMemcpyDeviceToDevice, E->stream);
            if (tlen > 0)
                cudaMemcpyAsync(trail + (size_t) b * trail_cap * H, E->trailing, sizeof(float) * tlen * H,
                                cudaMemcpyDeviceToDevice, E->stream);
            if (b == 0) {
                cudaMemcpyAsync(pad, E->pad, sizeof(float) * H, cudaMemcpyDeviceToDevice, E->stream);
                cudaMemcpyAsync(sp, E->sp, sizeof(SampleParams), cudaMemcpyDeviceToDevice, E->stream);
            }
            hs[b] = E->sess.st0;
            if (cudaStreamSynchronize(E->stream) != cudaSuccess || cudaGetLastError() != cudaSuccess) {
                err = "batch prefill copies"; return -1;
            }
            E->sess.active = false;
        }
        if (cudaMemcpy(st, hs.data(), sizeof(DevState) * n, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemset(d_err, 0, sizeof(int)) != cudaSuccess) {
            err = "batch state"; return -1;
        }
        B = n;
        produced.assign(n, 0);
        frames_ms = 0.0f;
        seq_frames = 0;
        if (graph_B != B && !capture()) return -1;
        (void) c;
        return 0;
    }

    // Runs up to n frames for the whole batch (stops early when every sequence is done).
    int run(int n) {
        if (B <= 0) { err = "no active batch"; return -1; }
        if (cudaEventRecord(ev0, stream) != cudaSuccess) { err = "event"; return -1; }
        for (int i = 0; i < n; ++i)
            if (cudaGraphLaunch(graph, stream) != cudaSuccess) { err = "graph launch"; return -1; }
        if (cudaEventRecord(ev1, stream) != cudaSuccess) { err = "event"; return -1; }
        std::vector<DevState> hs(B);
        int kerr = 0;
        if (cudaMemcpyAsync(hs.data(), st, sizeof(DevState) * B, cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
            cudaMemcpyAsync(&kerr, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) {
            err = "state readback"; return -1;
        }
        const cudaError_t e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) { err = std::string("batch frame: ") + cudaGetErrorString(e); return -1; }
        if (kerr) { err = "batch frame: a tensor-core GEMM wait timed out"; return -1; }
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ev0, ev1);
        frames_ms += ms;
        int adv = 0;
        for (int b = 0; b < B; ++b) {
            adv += hs[b].n_out - produced[b];
            produced[b] = hs[b].n_out;
        }
        seq_frames += adv;
        return adv;
    }

    // Runs n frames eagerly with events around every launch; ms_out[BC_N] and
    // launches_out[BC_N] per frame.
    bool profile(int n, float * ms_out, int * launches_out) {
        if (B <= 0) { err = "no active batch"; return false; }
        prof = true;
        prof_ev.clear();
        for (int i = 0; i < n; ++i) enqueue_frame();
        prof = false;
        if (cudaStreamSynchronize(stream) != cudaSuccess) { err = "profile frame"; return false; }
        for (int c = 0; c < BC_N; ++c) { ms_out[c] = 0.0f; launches_out[c] = 0; }
        for (auto & e : prof_ev) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, e.second.first, e.second.second);
            ms_out[e.first] += ms / n;
            launches_out[e.first] += 1;
            cudaEventDestroy(e.second.first);
            cudaEventDestroy(e.second.second);
        }
        for (int c = 0; c < BC_N; ++c) launches_out[c] /= n;
        prof_ev.clear();
        std::vector<DevState> hs(B);
        cudaMemcpy(hs.data(), st, sizeof(DevState) * B, cudaMemcpyDeviceToHost);
        for (int b = 0; b < B; ++b) produced[b] = hs[b].n_out;
        return true;
    }

    bool read_codes(int32_t * out, int32_t * nf) {
        std::vector<int> all((size_t) B * max_frames * NCB);
        if (cudaMemcpy(all.data(), codes, sizeof(int) * all.size(), cudaMemcpyDeviceToHost) != cudaSuccess) {
            err = "codes readback"; return false;
        }
        if (out) memcpy(out, all.data(), sizeof(int) * all.size());
        if (nf) for (int b = 0; b < B; ++b) nf[b] = produced[b];
        return true;
    }
};

}  // namespace qtts
