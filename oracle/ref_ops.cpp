// Op-level entry points into the reference's own code, for pinning the oracle.
// TEST INFRASTRUCTURE ONLY.
//
// This translation unit compiles the reference's src/nexterabert.cpp in place
// (the Makefile adds its directory to the include path; nothing is copied) and
// exposes its internal custom ops -- which live in an anonymous namespace --
// through plain C functions.  Data layouts at this boundary match oracle.h:
// activations are s8 = (u8 - 128) with scales [t][n_blk]; the wrappers convert
// to and from the reference's u8 + [t/4][n_blk][4] layout.  Together with
// ggml_shim.cpp the same library also exports the reference's whole C API
// (nextera_load / nextera_encode ...), so whole-model results can be compared.
#include "nexterabert.cpp"

#include <thread>

namespace {

// Runs a custom op the way ggml's graph executor does: fn(dst, ith, nth, ud)
// on nth threads that share the op's atomic work cursor.
void run_op(ggml_custom_op_t fn, ggml_tensor * dst, op_params * p, int nth) {
    if (nth <= 1) {
        fn(dst, 0, 1, p);
        return;
    }
    std::vector<std::thread> th;
    for (int i = 1; i < nth; ++i) th.emplace_back([=]() { fn(dst, i, nth, p); });
    fn(dst, 0, nth, p);
    for (auto & t : th) t.join();
}

ggml_tensor mk(const float * data, int64_t ne0, int64_t ne1) {
    ggml_tensor t;
    memset(&t, 0, sizeof t);
    t.type = GGML_TYPE_F32;
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = 1; t.ne[3] = 1;
    t.data = (void *) data;
    return t;
}

layout make_layout(const int32_t * lengths, int n) {
    layout l;
    l.build(lengths, n);
    return l;
}

int hw_threads() { return (int) std::max(1u, std::thread::hardware_concurrency()); }

// u8 + [t/4][n_blk][4] scales  ->  s8 + [t][n_blk] scales
void unpack_qact(const uint8_t * buf, int T, int C, int8_t * q, float * sx) {
    const int n_blk = (C + I8_BLOCK - 1) / I8_BLOCK;
    const float * s = (const float *) (buf + qact_scale_offset(T, C));
    for (size_t i = 0; i < (size_t) T * C; ++i) q[i] = (int8_t) ((int) buf[i] - NEXTERA_ACT_OFF);
    for (int t = 0; t < T; ++t) {
        for (int B = 0; B < n_blk; ++B) sx[(size_t) t * n_blk + B] = s[((size_t) (t / 4) * n_blk + B) * 4 + (t % 4)];
    }
}

std::vector<uint8_t> pack_qact(const int8_t * q, const float * sx, int T, int C) {
    const int n_blk = (C + I8_BLOCK - 1) / I8_BLOCK;
    std::vector<uint8_t> buf(qact_bytes(T, C, n_blk) + 64, 0);
    for (size_t i = 0; i < (size_t) T * C; ++i) buf[i] = (uint8_t) ((int) q[i] + NEXTERA_ACT_OFF);
    float * s = (float *) (buf.data() + qact_scale_offset(T, C));
    for (int t = 0; t < T; ++t) {
        for (int B = 0; B < n_blk; ++B) s[((size_t) (t / 4) * n_blk + B) * 4 + (t % 4)] = sx[(size_t) t * n_blk + B];
    }
    return buf;
}

// Runs a row op either as f32 output (q == NULL) or quantized (q, sx given).
void run_row_op(ggml_custom_op_t fn, ggml_tensor * dst_src, op_params * p, int C, int T, float * out,
                int8_t * q, float * sx) {
    if (!q) {
        dst_src->data = out;
        run_op(fn, dst_src, p, hw_threads());
        return;
    }
    p->quant = true;
    p->n_blk = (C + I8_BLOCK - 1) / I8_BLOCK;
    std::vector<uint8_t> buf(qact_bytes(T, C, p->n_blk) + 64, 0);
    dst_src->data = buf.data();
    run_op(fn, dst_src, p, hw_threads());
    unpack_qact(buf.data(), T, C, q, sx);
}

} // namespace

extern "C" {

NEXTERA_API int ref_act_max(void) { return NEXTERA_ACT_MAX; }

NEXTERA_API void ref_build_i8_weight(int type, const void * data, int n_in, int n_out,
                                     int8_t * w, float * scale, int32_t * off) {
    i8_weight iw;
    build_i8_weight(iw, (ggml_type) type, data, n_in, n_out, hw_threads());
    memcpy(w, iw.w.data(), iw.w.size());
    memcpy(scale, iw.scale.data(), sizeof(float) * iw.scale.size());
    memcpy(off, iw.off.data(), sizeof(int32_t) * iw.off.size());
}

// op_copy: f32 rows -> quantized (quantize_row)
NEXTERA_API void ref_quantize_rows(const float * x, int T, int C, int8_t * q, float * sx) {
    ggml_tensor src = mk(x, C, T), dst = mk(nullptr, C, T);
    dst.src[0] = &src;
    op_params p;
    run_row_op(op_copy, &dst, &p, C, T, nullptr, q, sx);
}

NEXTERA_API void ref_linear_i8(const int8_t * xq, const float * sx, int T, const int8_t * w, const float * sw,
                               const int32_t * off, int n_in, int n_out, const float * res, float * out) {
    i8_weight iw;
    iw.n_in = n_in;
    iw.n_out = n_out;
    iw.n_blk = (n_in + I8_BLOCK - 1) / I8_BLOCK;
    iw.w.assign(w, w + (size_t) n_in * n_out);
    iw.scale.assign(sw, sw + (size_t) iw.n_blk * n_out);
    iw.off.assign(off, off + (size_t) iw.n_blk * n_out);
    std::vector<uint8_t> qb = pack_qact(xq, sx, T, n_in);
    ggml_tensor a = mk((const float *) qb.data(), 1, 1), r = mk(res, n_out, T), dst = mk(out, n_out, T);
    dst.src[0] = &a;
    dst.src[1] = res ? &r : nullptr;
    op_params p;
    p.i8 = &iw;
    p.n_rows = T;
    p.residual = res != nullptr;
    run_op(op_linear_i8, &dst, &p, hw_threads());
}

NEXTERA_API void ref_rms_norm(const float * x, const float * gain, float eps, int T, int C, float * out,
                              int8_t * q, float * sx) {
    ggml_tensor src = mk(x, C, T), dst = mk(nullptr, C, T);
    dst.src[0] = &src;
    op_params p;
    p.gain = gain;
    p.eps = eps;
    run_row_op(op_rms_norm, &dst, &p, C, T, out, q, sx);
}

NEXTERA_API void ref_relu_sqr(const float * x, int T, int C, float * out, int8_t * q, float * sx) {
    ggml_tensor src = mk(x, C, T), dst = mk(nullptr, C, T);
    dst.src[0] = &src;
    op_params p;
    run_row_op(op_relu_sqr, &dst, &p, C, T, out, q, sx);
}

NEXTERA_API void ref_gate(const float * g, const float * y, int T, int C, float * out, int8_t * q, float * sx) {
    ggml_tensor a = mk(g, C, T), b = mk(y, C, T), dst = mk(nullptr, C, T);
    dst.src[0] = &a;
    dst.src[1] = &b;
    op_params p;
    run_row_op(op_gate, &dst, &p, C, T, out, q, sx);
}

NEXTERA_API void ref_dwconv(const float * x, const float * r, const float * taps, int k,
                            const int32_t * lengths, int n_docs, int C, float * out, int8_t * q, float * sx) {
    layout lay = make_layout(lengths, n_docs);
    const int T = lay.total;
    ggml_tensor a = mk(x, C, T), b = mk(r, C, T), dst = mk(nullptr, C, T);
    dst.src[0] = &a;
    dst.src[1] = r ? &b : nullptr;
    op_params p;
    p.lay = &lay;
    p.taps = taps;
    p.k = k;
    run_row_op(op_dwconv, &dst, &p, C, T, out, q, sx);
}

NEXTERA_API void ref_lily_state(const float * a, const float * x, const float * b, const float * taps, int k,
                                const int32_t * lengths, int n_docs, int C, float * out, int8_t * q, float * sx) {
    layout lay = make_layout(lengths, n_docs);
    const int T = lay.total;
    ggml_tensor ta = mk(a, C, T), tx = mk(x, C, T), tb = mk(b, C, T), dst = mk(nullptr, C, T);
    dst.src[0] = &ta;
    dst.src[1] = &tx;
    dst.src[2] = &tb;
    op_params p;
    p.lay = &lay;
    p.taps = taps;
    p.k = k;
    run_row_op(op_lily_state, &dst, &p, C, T, out, q, sx);
}

NEXTERA_API void ref_qk_prep(const float * x, const float * alpha, const float * beta, float base,
                             const int32_t * lengths, int n_docs, int H, int D, int head_major, float * out) {
    layout lay = make_layout(lengths, n_docs);
    const int T = lay.total;
    int max_len = 0;
    for (int i = 0; i < n_docs; ++i) max_len = std::max(max_len, lengths[i]);
    rope_table rope;
    build_rope(rope, max_len, base, D);
    ggml_tensor src = mk(x, (int64_t) H * D, T), dst = mk(out, (int64_t) H * D, T);
    dst.src[0] = &src;
    op_params p;
    p.lay = &lay;
    p.alpha = alpha;
    p.beta = beta;
    p.rope = &rope;
    p.head_dim = D;
    p.head_major = head_major != 0;
    run_op(op_qk_prep, &dst, &p, hw_threads());
}

NEXTERA_API void ref_rope_table(int n_pos, float base, int head_dim, float * cos_t, float * sin_t) {
    rope_table rope;
    build_rope(rope, n_pos, base, head_dim);
    memcpy(cos_t, rope.cos.data(), sizeof(float) * rope.cos.size());
    memcpy(sin_t, rope.sin.data(), sizeof(float) * rope.sin.size());
}

NEXTERA_API void ref_head_major(const float * x, int T, int H, int D, float * out) {
    ggml_tensor src = mk(x, (int64_t) H * D, T), dst = mk(out, (int64_t) H * D, T);
    dst.src[0] = &src;
    op_params p;
    p.head_dim = D;
    run_op(op_head_major, &dst, &p, hw_threads());
}

NEXTERA_API void ref_block_mean(const float * h, const float * g, int C, int block,
                                const int32_t * lengths, int n_docs, float * out, int8_t * q, float * sx) {
    layout lay = make_layout(lengths, n_docs);
    std::vector<int32_t> nb(n_docs);
    for (int i = 0; i < n_docs; ++i) nb[i] = (lengths[i] + block - 1) / block;
    layout blay = make_layout(nb.data(), n_docs);
    ggml_tensor th = mk(h, C, lay.total), tg = mk(g, C, lay.total), dst = mk(nullptr, C, blay.total);
    dst.src[0] = &th;
    dst.src[1] = g ? &tg : nullptr;
    op_params p;
    p.lay = &lay;
    p.blay = &blay;
    p.block = block;
    run_row_op(op_block_mean, &dst, &p, C, blay.total, out, q, sx);
}

NEXTERA_API void ref_upsample_add(const float * y, const float * r, int C, int block,
                                  const int32_t * lengths, int n_docs, float * out) {
    layout lay = make_layout(lengths, n_docs);
    std::vector<int32_t> nb(n_docs);
    for (int i = 0; i < n_docs; ++i) nb[i] = (lengths[i] + block - 1) / block;
    layout blay = make_layout(nb.data(), n_docs);
    ggml_tensor ty = mk(y, C, blay.total), tr = mk(r, C, lay.total), dst = mk(out, C, lay.total);
    dst.src[0] = &ty;
    dst.src[1] = &tr;
    op_params p;
    p.lay = &lay;
    p.blay = &blay;
    p.block = block;
    run_op(op_upsample_add, &dst, &p, hw_threads());
}

// q [T][H*D] row-major; k, v head-major [G][T][D]; scale per document
NEXTERA_API void ref_attention(const float * q, const float * k, const float * v, int H, int G, int D, int half,
                               const float * scale, const int32_t * lengths, int n_docs, float * out) {
    layout lay = make_layout(lengths, n_docs);
    const int T = lay.total;
    ggml_tensor tq = mk(q, (int64_t) H * D, T), tk = mk(k, (int64_t) G * D, T), tv = mk(v, (int64_t) G * D, T);
    ggml_tensor dst = mk(out, (int64_t) H * D, T);
    dst.src[0] = &tq;
    dst.src[1] = &tk;
    dst.src[2] = &tv;
    op_params p;
    p.lay = &lay;
    p.head_dim = D;
    p.n_head = H;
    p.n_kv_head = G;
    p.half = half;
    p.scale.assign(scale, scale + n_docs);
    run_op(op_attention, &dst, &p, hw_threads());
}

} // extern "C"
