// batch_host.cuh — host side of the batched frame loop (included into
// engine.cu after the Engine definition; kernels in batch_engine.cuh).
#pragma once

namespace qtts {

struct TiledLayer {
    uint8_t * qkv = nullptr, * o = nullptr, * gu = nullptr, * down = nullptr;
    __half * sqkv = nullptr, * so = nullptr, * sgu = nullptr, * sdown = nullptr;   // Q8_0 block scales (q8_s_off)
};

// A weight matrix (or a gate/up pair, interleaved in 64-row groups) copied
// into the canonical tcgen05 tile layout of k_gemm_tc.
inline bool tile_check(const DMat & W, const DMat * W2, std::string & err) {
    const int rows_w = W2 ? 2 * W.rows : W.rows;
    if (W.type != W_F16) { err = "tensor-core path: F16 weights only"; return false; }
    if (rows_w % TC_BM || W.cols % TC_BK || (W2 && W.rows % (TC_BM / 2))) { err = "tensor-core path: matrix shape"; return false; }
    return true;
}
inline bool tile_launch(const DMat & W, const DMat * W2, uint8_t * out, cudaStream_t stream) {
    const int rows_w = W2 ? 2 * W.rows : W.rows;
    k_tile_weights<<<rows_w, 128, 0, stream>>>((const __half *) W.w, W2 ? (const __half *) W2->w : nullptr, rows_w,
                                              W.cols, out);
    return cudaGetLastError() == cudaSuccess;
}

// Pack (RMSNorm, F16 / hi-lo) + tcgen05 GEMM for m activation rows on `stream`
// (shared by the batched frame and the tensor-core prefill).  xin == nullptr:
// the activation tiles are already in xt2 (written by the producer).  xt_next:
// SwiGLU only, also write h as hi/lo tiles into xt2 for the down GEMM.
struct TcGemm {
    cudaStream_t stream = nullptr;
    uint8_t * xt = nullptr, * xt2 = nullptr;
    int * d_err = nullptr;
    float eps = 0.0f;
    int ldxn = 0;
    int launches = 0;
    void pack(const float * xin, int ldx, int m, int np, int cols, const float * norm, int act, float * xn_out) {
        PackArgs pa{};
        pa.x = xin; pa.ldx = ldx; pa.m_real = m; pa.np = np; pa.cols = cols; pa.gain = norm;
        pa.eps = eps; pa.act = act; pa.out = xt; pa.xn_out = xn_out; pa.ldxn = ldxn;
        pdl_launch(k_pack_act, dim3(act == TC_ACT_SPLIT ? np / 2 : np), dim3(256), 0, stream, pa);
        launches += 1;
    }
    void gemm(const uint8_t * wt, int rows_w, int cols, const uint8_t * xsrc, int m, int np, int act, int epi,
              float * y, int ldy, const float * resid, bool xt_next, int mp) {
        GemmTcArgs g{};
        g.w = wt; g.x = xsrc; g.rows_w = rows_w; g.cols = cols; g.np = np; g.m_real = m;
        g.split = act == TC_ACT_SPLIT; g.epi = epi; g.y = y; g.ldy = ldy; g.resid = resid; g.ldr = ldy; g.err = d_err;
        if (xt_next) { g.xt_out = xt2; g.xt_np = 2 * mp; }
        g.ksplit = tc_choose_split(g);
        tc_launch(g, stream);
        launches += 1;
    }
};

// Q8_0 projection of m F32 rows on the tensor cores: quantise the rows per
// 32-block into xq / xqs (k_pack_q8, optional RMSNorm), then the kind::i8 GEMM.
// Returns the number of launches.
inline int q8_project(cudaStream_t stream, uint8_t * xq, float * xqs, int * d_err, float eps, const uint8_t * wt,
                      const __half * ws, int rows_w, int cols, const float * xin, int ldx, int m, const float * norm,
                      int epi, float * y, int ldy, const float * resid) {
    const int mp = (m + 15) / 16 * 16;
    PackQ8Args pa{};
    pa.x = xin; pa.ldx = ldx; pa.m_real = m; pa.np = mp; pa.cols = cols; pa.gain = norm;
    pa.eps = eps; pa.out = xq; pa.dscale = xqs;
    pdl_launch(k_pack_q8, dim3(mp), dim3(256), 0, stream, pa);
    GemmQ8Args g{};
    g.w = wt; g.ws = ws; g.x = xq; g.xs = xqs; g.rows_w = rows_w; g.cols = cols; g.np = mp; g.m_real = m;
    g.epi = epi; g.y = y; g.ldy = ldy; g.resid = resid; g.ldr = ldy; g.err = d_err;
    g.ksplit = q8_choose_split(g);
    q8_launch(g, stream);
    return 2;
}

// Tiles of a Q8_0 matrix (or gate/up pair) and its block scales for k_gemm_q8.
inline bool tile_q8_check(const DMat & W, const DMat * W2, std::string & err) {
    const int rows_w = W2 ? 2 * W.rows : W.rows;
    if (W.type != W_Q8_0 || rows_w % TC_BM || W.cols % Q8_BK || (W2 && W.rows % (TC_BM / 2))) {
        err = "Q8_0 tensor-core path: matrix shape"; return false;
    }
    return true;
}

struct BatchEngine {
    Engine * E = nullptr;
    int dev = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    int Bmax = 0, B = 0, n_max = 0, max_frames = 0, max_pages = 0, n_pages = 0, trail_cap = 0;
    int H = 0, NH = 0, NKV = 0, QD = 0, KD = 0, QKVD = 0, FF = 0, CFF = 0, V0 = 0, V1 = 0, NCB = 0;
    std::vector<TiledLayer> TL, TCP;
    bool q8 = false;   // Q8_0 layer weights: projections as kind::i8 tcgen05 GEMMs (heads stay F16 tcgen05)
    uint8_t * xq = nullptr;                 // Q8_0 activation tiles
    float * xqs = nullptr;                  // their block scales
    std::vector<uint8_t *> cp_head_t;
    uint8_t * codec_head_t = nullptr;
    std::vector<void *> owned;
    float * x = nullptr, * xcp = nullptr, * qkv = nullptr, * att = nullptr, * hbuf = nullptr;
    float * logits = nullptr, * cp_logits = nullptr, * hidden = nullptr, * trail = nullptr, * pad = nullptr;
    uint8_t * xt = nullptr, * xt2 = nullptr;   // tiled activations: pack target / producer-written
    DevState * st = nullptr;
    SampleParams * sp = nullptr;
    int * codes = nullptr, * page_table = nullptr, * d_err = nullptr;
    int * d_max_len = nullptr;              // per-sequence frame budget (k_frame_end_batch stops a sequence there)
    std::vector<int> max_len;
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

    bool tile_q8(const DMat & W, const DMat * W2, uint8_t ** out, __half ** sout) {
        const int rows_w = W2 ? 2 * W.rows : W.rows;
        if (!tile_q8_check(W, W2, err)) return false;
        if (!alloc(out, (size_t) rows_w * W.cols) || !alloc(sout, (size_t) rows_w * (W.cols / 32) * 2)) return false;
        k_tile_q8<<<rows_w, 128, 0, stream>>>(W, W2 ? *W2 : DMat{}, rows_w, *out, *sout);
        return cudaGetLastError() == cudaSuccess;
    }
    bool tile(const DMat & W, const DMat * W2, uint8_t ** out) {
        if (!tile_check(W, W2, err)) return false;
        if (!alloc(out, (size_t)(W2 ? 2 * W.rows : W.rows) * W.cols * 2)) return false;
        return tile_launch(W, W2, *out, stream);
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
        auto tq = [&](std::vector<LayerW> & Ls, std::vector<TiledLayer> & T) {
            for (size_t i = 0; i < Ls.size(); ++i)
                if (!tile_q8(Ls[i].qkv, nullptr, &T[i].qkv, &T[i].sqkv) || !tile_q8(Ls[i].o, nullptr, &T[i].o, &T[i].so) ||
                    !tile_q8(Ls[i].gate, &Ls[i].up, &T[i].gu, &T[i].sgu) ||
                    !tile_q8(Ls[i].down, nullptr, &T[i].down, &T[i].sdown))
                    return false;
            return true;
        };
        q8 = E->L[0].qkv.type == W_Q8_0;
        if (!q8 && (!tl(E->L, TL) || !tl(E->CPL, TCP))) return false;
        if (q8 && (!tq(E->L, TL) || !tq(E->CPL, TCP))) return false;
        if (q8 && 2 * bmax > Q8_MAX_N) { err = "Q8_0 batches: max_batch must be <= 64"; return false; }
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
            !alloc(&codes, sizeof(int) * Bmax * max_frames * NCB) || !alloc(&d_err, sizeof(int)) ||
            !alloc(&xq, (size_t) Q8_MAX_N * maxc) || !alloc(&xqs, sizeof(float) * Q8_MAX_N * (maxc / 32)) ||
            !alloc(&d_max_len, sizeof(int) * Bmax))
            return false;
        trail_cap = 1024;
        if (!alloc(&trail, sizeof(float) * Bmax * trail_cap * H)) return false;
        max_pages = (n_max + BP_PAGE - 1) / BP_PAGE;
        n_pages = Bmax * max_pages;
        if (!alloc(&pool, sizeof(__half) * bp_page_elems((int) E->L.size(), NKV) * n_pages) ||
            !alloc(&page_table, sizeof(int) * Bmax * max_pages) ||
            !alloc(&attn_part, sizeof(float) * Bmax * NKV * PA_MAX_SPLIT * (NH / NKV) * PA_PART))
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
            q8_set_attributes() != cudaSuccess ||
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
        TcGemm t{stream, xt, xt2, d_err, E->cfg.rms_norm_eps, H, 0};
        if (xin) {
            pb(BC_PACK);
            t.pack(xin, ldx, m, np, cols, norm, act, xn_out);
            pe();
        }
        pb(gemm_cls);
        t.gemm(wt, rows_w, cols, xin ? xt : xt2, m, np, act, epi, y, ldy, resid, xt_next, mp);
        pe();
        launches += t.launches;
    }
    int gemm_cls = BC_GEMM_QKV;

    // Q8_0 projection of m F32 rows on the tensor cores: quantise the rows per
    // 32-block (k_pack_q8, optional RMSNorm) and run the kind::i8 GEMM.
    void gemm_q8(const uint8_t * wt, const __half * ws, int rows_w, int cols, const float * xin, int ldx, int m,
                 const float * norm, int epi, float * y, int ldy, const float * resid) {
        pb(gemm_cls);
        launches += q8_project(stream, xq, xqs, d_err, E->cfg.rms_norm_eps, wt, ws, rows_w, cols, xin, ldx, m, norm, epi,
                               y, ldy, resid);
        pe();
    }

    // One decoder layer's four projections over `rows` rows of X: tcgen05 GEMMs
    // (F16) or 8-row GEMV chunks (Q8_0).  which: 0 q|k|v, 1 O (+ residual),
    // 2 gate/up (SwiGLU), 3 down (+ residual).
    void proj(int which, const LayerW & l, const TiledLayer & t, float * X, int rows, int ffn) {
        const int cols_o = QD;
        switch (which) {
            case 0:
                gemm_cls = BC_GEMM_QKV;
                if (q8) gemm_q8(t.qkv, t.sqkv, QKVD, H, X, H, rows, l.attn_norm, TC_EPI_STORE, qkv, QKVD, nullptr);
                else gemm(t.qkv, QKVD, H, X, H, rows, l.attn_norm, TC_ACT_F16, TC_EPI_STORE, qkv, QKVD, nullptr);
                break;
            case 1:
                gemm_cls = BC_GEMM_O;
                if (q8) gemm_q8(t.o, t.so, H, cols_o, att, cols_o, rows, nullptr, TC_EPI_RESID, X, H, X);
                else gemm(t.o, H, QD, nullptr, QD, rows, nullptr, TC_ACT_F16, TC_EPI_RESID, X, H, X);
                break;
            case 2:
                gemm_cls = BC_GEMM_GU;
                if (q8) gemm_q8(t.gu, t.sgu, 2 * ffn, H, X, H, rows, l.ffn_norm, TC_EPI_SWIGLU, hbuf, ffn, nullptr);
                else gemm(t.gu, 2 * ffn, H, X, H, rows, l.ffn_norm, TC_ACT_F16, TC_EPI_SWIGLU, hbuf, ffn, nullptr, nullptr, true);
                break;
            default:
                gemm_cls = BC_GEMM_DOWN;
                if (q8) gemm_q8(t.down, t.sdown, H, ffn, hbuf, ffn, rows, nullptr, TC_EPI_RESID, X, H, X);
                else gemm(t.down, H, ffn, nullptr, ffn, rows, nullptr, TC_ACT_SPLIT, TC_EPI_RESID, X, H, X);
                break;
        }
    }

    void cp_layers(int M, bool f32, int pos_static) {
        const int rows = B * M;
        for (size_t il = 0; il < E->CPL.size(); ++il) {
            const LayerW & l = E->CPL[il];
            const TiledLayer t = TCP[il];
            proj(0, l, t, xcp, rows, CFF);
            FusedAttn fa{};
            fa.qkv = qkv; fa.ldq = QKVD; fa.n_heads = NH; fa.n_kv_heads = NKV; fa.q_norm = l.q_norm;
            fa.k_norm = l.k_norm; fa.eps = E->cfg.rms_norm_eps; fa.rope = E->rope_cp;
            fa.kc = cpk + il * cp_layer; fa.vc = cpv + il * cp_layer; fa.pos_static = pos_static; fa.M = M;
            fa.f32_mode = f32 ? 1 : 0; fa.scale = 1.0f / sqrtf((float) QTTS_HD); fa.out = att; fa.ldo = QD;
            fa.xt = q8 ? nullptr : xt2; fa.xt_np = (rows + 15) / 16 * 16;
            pb(BC_ATTN_CP);
            pdl_launch(k_cp_attn_warp, dim3((B * NH * M + CPW_WARPS - 1) / CPW_WARPS), dim3(CPW_WARPS * 32), 0, stream, fa,
                       cp_stride, (const DevState *) st, B);
            pe();
            proj(1, l, t, xcp, rows, CFF);
            proj(2, l, t, xcp, rows, CFF);
            proj(3, l, t, xcp, rows, CFF);
            launches += 1;
        }
    }

    // Page ranges per (sequence, kv head) of the talker attention: QTTS_ATTN_SPLIT,
    // else 1 when the (sequence, kv head) CTAs alone cover the SMs or the capacity
    // is below 1024 positions, else enough ranges to give every SM two CTAs (at
    // most 16, at most the pages).
    float * attn_part = nullptr;
    int attn_split(int b) const {
        int ns = 1;
        if (const char * e = getenv("QTTS_ATTN_SPLIT")) ns = atoi(e);
        else if (n_max >= 1024 && b * NKV < E->n_sm) ns = (2 * E->n_sm + b * NKV - 1) / (b * NKV);
        return std::max(1, std::min(std::min(ns, PA_MAX_SPLIT), max_pages));
    }

    void talker_layers() {
        const int G = NH / NKV;
        for (size_t il = 0; il < E->L.size(); ++il) {
            const LayerW & l = E->L[il];
            const TiledLayer t = TL[il];
            proj(0, l, t, x, B, FF);
            PagedAttnArgs pa{};
            pa.qkv = qkv; pa.ldq = QKVD; pa.n_heads = NH; pa.n_kv_heads = NKV; pa.n_layers = (int) E->L.size();
            pa.layer = (int) il; pa.q_norm = l.q_norm; pa.k_norm = l.k_norm; pa.eps = E->cfg.rms_norm_eps;
            pa.rope = rope_t; pa.pool = pool; pa.page_table = page_table; pa.max_pages = max_pages; pa.st = st;
            pa.scale = 1.0f / sqrtf((float) QTTS_HD); pa.out = att; pa.ldo = QD; pa.n_max = n_max;
            pa.xt = q8 ? nullptr : xt2; pa.xt_np = (B + 15) / 16 * 16;
            // split-KV over page ranges when (sequence, kv head) pairs alone leave SMs idle
            const int ns = attn_split(B);
            pa.nsplit = ns;
            pa.part = attn_part;
            const int chunk = (max_pages + ns - 1) / ns;
            pa.n_max = std::min(n_max, chunk * BP_PAGE);
            pb(BC_ATTN_TALKER);
            pdl_launch(k_attn_paged, dim3(B * NKV * ns), dim3(PA_BLOCK), paged_attn_smem(pa.n_max, G), stream, pa);
            if (ns > 1) pdl_launch(k_attn_combine, dim3(B * NKV), dim3(QTTS_HD), 0, stream, pa);
            pe();
            if (ns > 1) launches += 1;
            proj(1, l, t, x, B, FF);
            proj(2, l, t, x, B, FF);
            proj(3, l, t, x, B, FF);
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
        pdl_launch(k_frame_end_batch, dim3((B + 127) / 128), dim3(128), 0, stream, st, B, (const int *) d_max_len);
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
        max_len.assign(n, 0);
        for (int b = 0; b < n; ++b) {
            if (ps[b].max_len < 1 || ps[b].max_len > max_frames) { err = "max_len must be in [1, max_frames]"; return -1; }
            max_len[b] = ps[b].max_len;
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
            cudaMemcpy(d_max_len, max_len.data(), sizeof(int) * n, cudaMemcpyHostToDevice) != cudaSuccess ||
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

    // Runs up to n frames for the whole batch (stops early when every sequence is
    // done).  n is clamped to the largest remaining budget (max_len - produced);
    // sequences with smaller budgets stop on the device at their own max_len.
    int run(int n) {
        if (B <= 0) { err = "no active batch"; return -1; }
        int left = 0;
        for (int b = 0; b < B; ++b) left = std::max(left, max_len[b] - produced[b]);
        n = std::max(0, std::min(n, left));
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

// Tensor-core talker prefill (F16 weights): forward_prefill over up to
// PREFILL_TC_ROWS prompt rows per call with the batched path's tcgen05 GEMMs
// (weights tiled once, on first use), the prefill attention kernels and the
// engine's KV cache.  Per layer: pack+GEMM q|k|v, q/k norm + RoPE + KV append,
// causal attention, GEMM O (+ residual), pack+GEMM gate/up (SwiGLU, h written
// as hi/lo tiles), GEMM down (+ residual).
struct PrefillTC {
    Engine * E = nullptr;
    std::string err;
    std::vector<TiledLayer> TL;
    std::vector<void *> owned;
    float * qkv = nullptr, * att = nullptr, * hbuf = nullptr;
    uint8_t * xt = nullptr, * xt2 = nullptr;
    int * d_err = nullptr;
    bool q8 = false;                        // Q8_0 weights: kind::i8 GEMMs
    uint8_t * xq = nullptr;
    float * xqs = nullptr;

    template <class T>
    bool alloc(T ** p, size_t bytes) {
        if (cudaMalloc(p, bytes) != cudaSuccess) { err = "prefill: out of device memory"; return false; }
        owned.push_back(*p);
        return true;
    }
    ~PrefillTC() { for (void * p : owned) cudaFree(p); }

    bool tile(const DMat & W, const DMat * W2, uint8_t ** out) {
        if (!tile_check(W, W2, err)) return false;
        if (!alloc(out, (size_t)(W2 ? 2 * W.rows : W.rows) * W.cols * 2)) return false;
        return tile_launch(W, W2, *out, E->stream);
    }

    bool create(Engine * eng) {
        E = eng;
        const qtts_config & c = eng->cfg;
        const int R = PREFILL_TC_ROWS, H = c.hidden_size, QD = eng->QD(), FF = c.intermediate_size;
        TL.resize(E->L.size());
        q8 = E->L[0].qkv.type == W_Q8_0;
        auto tq = [&](const DMat & W, const DMat * W2, uint8_t ** out, __half ** sout) {
            const int rows_w = W2 ? 2 * W.rows : W.rows;
            if (!tile_q8_check(W, W2, err)) return false;
            if (!alloc(out, (size_t) rows_w * W.cols) || !alloc(sout, (size_t) rows_w * (W.cols / 32) * 2)) return false;
            k_tile_q8<<<rows_w, 128, 0, E->stream>>>(W, W2 ? *W2 : DMat{}, rows_w, *out, *sout);
            return cudaGetLastError() == cudaSuccess;
        };
        for (size_t i = 0; i < E->L.size(); ++i) {
            LayerW & l = E->L[i];
            TiledLayer & t = TL[i];
            const bool ok = q8 ? tq(l.qkv, nullptr, &t.qkv, &t.sqkv) && tq(l.o, nullptr, &t.o, &t.so) &&
                                     tq(l.gate, &l.up, &t.gu, &t.sgu) && tq(l.down, nullptr, &t.down, &t.sdown)
                               : tile(l.qkv, nullptr, &t.qkv) && tile(l.o, nullptr, &t.o) && tile(l.gate, &l.up, &t.gu) &&
                                     tile(l.down, nullptr, &t.down);
            if (!ok) return false;
        }
        const int maxc = std::max(std::max(H, QD), FF);
        if (q8 && (!alloc(&xq, (size_t) Q8_MAX_N * maxc) || !alloc(&xqs, sizeof(float) * Q8_MAX_N * (maxc / 32))))
            return false;
        if (q8 && q8_set_attributes() != cudaSuccess) { err = "prefill: kernel attributes"; return false; }
        if (!alloc(&qkv, sizeof(float) * R * eng->QKVD()) || !alloc(&att, sizeof(float) * R * QD) ||
            !alloc(&hbuf, sizeof(float) * R * FF) || !alloc(&xt, (size_t) TC_MAX_N * maxc * 2) ||
            !alloc(&xt2, (size_t) TC_MAX_N * maxc * 2) || !alloc(&d_err, sizeof(int)))
            return false;
        if (cudaMemsetAsync(d_err, 0, sizeof(int), E->stream) != cudaSuccess) { err = "prefill: memset"; return false; }
        if (cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 201 * 1024) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
            err = "prefill: kernel attributes"; return false;
        }
        return true;
    }

    // All talker layers over rows X[M][H] at positions n_past .. n_past + M - 1.
    bool layers(float * X, int M, int n_past) {
        const qtts_config & c = E->cfg;
        const int H = c.hidden_size, QD = E->QD(), QKVD = E->QKVD(), FF = c.intermediate_size;
        const int G = c.n_attention_heads / c.n_key_value_heads;
        if (M < 1 || M > PREFILL_TC_ROWS) { err = "prefill: chunk size"; return false; }
        const size_t layer_elems = (size_t) E->n_ctx * c.n_key_value_heads * QTTS_HD;
        const size_t att_smem = attn_smem_bytes(E->n_ctx, G);
        const int mp = (M + 15) / 16 * 16;
        TcGemm t{E->stream, xt, xt2, d_err, c.rms_norm_eps, H, 0};
        for (size_t il = 0; il < E->L.size(); ++il) {
            const LayerW & l = E->L[il];
            const TiledLayer & w = TL[il];
            if (q8) {
                const float eps = c.rms_norm_eps;
                int n = q8_project(E->stream, xq, xqs, d_err, eps, w.qkv, w.sqkv, QKVD, H, X, H, M, l.attn_norm,
                                   TC_EPI_STORE, qkv, QKVD, nullptr);
                E->prefill_attention(l, E->kc + il * layer_elems, E->vc + il * layer_elems, E->rope_t, qkv, QKVD, M,
                                     nullptr, n_past, nullptr, att, QD, nullptr, 0, att_smem);
                n += q8_project(E->stream, xq, xqs, d_err, eps, w.o, w.so, H, QD, att, QD, M, nullptr, TC_EPI_RESID, X,
                                H, X);
                n += q8_project(E->stream, xq, xqs, d_err, eps, w.gu, w.sgu, 2 * FF, H, X, H, M, l.ffn_norm,
                                TC_EPI_SWIGLU, hbuf, FF, nullptr);
                n += q8_project(E->stream, xq, xqs, d_err, eps, w.down, w.sdown, H, FF, hbuf, FF, M, nullptr,
                                TC_EPI_RESID, X, H, X);
                E->launches += n;
                continue;
            }
            t.pack(X, H, M, mp, H, l.attn_norm, TC_ACT_F16, nullptr);
            t.gemm(w.qkv, QKVD, H, xt, M, mp, TC_ACT_F16, TC_EPI_STORE, qkv, QKVD, nullptr, false, mp);
            E->prefill_attention(l, E->kc + il * layer_elems, E->vc + il * layer_elems, E->rope_t, qkv, QKVD, M,
                                 nullptr, n_past, nullptr, att, QD, nullptr, 0, att_smem);
            t.pack(att, QD, M, mp, QD, nullptr, TC_ACT_F16, nullptr);
            t.gemm(w.o, H, QD, xt, M, mp, TC_ACT_F16, TC_EPI_RESID, X, H, X, false, mp);
            t.pack(X, H, M, mp, H, l.ffn_norm, TC_ACT_F16, nullptr);
            t.gemm(w.gu, 2 * FF, H, xt, M, mp, TC_ACT_F16, TC_EPI_SWIGLU, hbuf, FF, nullptr, true, mp);
            // ffn_down: F32 activation (F16 weight cast to F32 by the reference) as F16 hi + lo
            t.gemm(w.down, H, FF, xt2, M, 2 * mp, TC_ACT_SPLIT, TC_EPI_RESID, X, H, X, false, mp);
        }
        E->launches += t.launches;
        if (cudaGetLastError() != cudaSuccess) { err = "prefill: launch failed"; return false; }
        return true;
    }
};

bool prefill_tc_layers(Engine & E, float * X, int M, int n_past) {
    if (!E.ptc) {
        PrefillTC * p = new PrefillTC();
        if (!p->create(&E)) { E.err = p->err; delete p; return false; }
        E.ptc = p;
    }
    if (!E.ptc->layers(X, M, n_past)) { E.err = E.ptc->err; return false; }
    return true;
}

bool prefill_tc_check(Engine & E) {
    int e = 0;
    if (!E.ptc || cudaMemcpy(&e, E.ptc->d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess || e != 0) {
        E.err = "prefill: tensor-core GEMM error " + std::to_string(e);
        return false;
    }
    return true;
}

void prefill_tc_free(PrefillTC * p) { delete p; }

}  // namespace qtts
