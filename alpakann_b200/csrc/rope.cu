// rope.cu -- rope / ropeInPlace (reference: onHost/nn/rope.hpp:21-135,
// onAcc/internal/nn/rope.hpp:15-49).
//
// Interleaved-pair rotation: for pair p of a head vector,
//   x'[2p]   = x[2p] * cos - x[2p+1] * sin
//   x'[2p+1] = x[2p] * sin + x[2p+1] * cos
// with cos/sin = table[positionOffset + token][p].
//
// The reference's ropeInPlace allocates a temporary, launches one kernel per
// element into it and copies back, per tensor (rope.hpp:96-135). Here one
// launch rotates Q and K together, truly in place: each thread owns whole
// pairs (two pairs = one 16-byte vector in fp32, one pair in fp64), reads them
// and writes them back. Products and sums are left uncontracted (no FMA), so
// the result is bit-identical to the reference expression evaluated in order.
//
// kvCacheAppend writes a decode step's new K/V rows (BTHD) into BHTD caches at
// a position -- the helper on either side of the attention path in a decoder
// layer (one layer of an LBHTD cache, core/layout.hpp:41-45, is a BHTD view) --
// optionally rotating K on the way, with the same expression as ropeInPlace.
#include "common.cuh"
#include "reduce.cuh"

namespace ann {
namespace {

struct RopeJob {
    const void* in;
    void* out;
    int64_t e0, e1, e2;    // leading extents
    int64_t npv;           // pair-vectors per head vector
    int64_t si[4], so[4];  // element strides
    int64_t items;         // e0 * e1 * e2 * npv
    int rotate;            // 0: copy the pairs unchanged
};

struct RopeArgs {
    RopeJob job[2];
    int njobs;
    const void* cos;
    const void* sin;
    int64_t cs0, cs1, ss0, ss1;
    int layout;
    int64_t pos_off;
};

template <typename T, int PV, bool VEC>  // PV pairs per work item; 2*PV contiguous elements when VEC
__device__ __forceinline__ void rope_item(RopeArgs const& a, RopeJob const& j, int64_t flat) {
    T const* cosT = static_cast<T const*>(a.cos);
    T const* sinT = static_cast<T const*>(a.sin);
    int64_t const pv = flat % j.npv;
    int64_t r = flat / j.npv;
    int64_t const a2 = r % j.e2;
    r /= j.e2;
    int64_t const a1 = r % j.e1;
    int64_t const a0 = r / j.e1;
    int64_t const tok = a.layout == ANN_LAYOUT_BTHD ? a1 : a2;
    int64_t const pos = a.pos_off + tok;
    T const* in = static_cast<T const*>(j.in) + a0 * j.si[0] + a1 * j.si[1] + a2 * j.si[2];
    T* out = static_cast<T*>(j.out) + a0 * j.so[0] + a1 * j.so[1] + a2 * j.so[2];
    T x[2 * PV];
    if constexpr (VEC) {
        using V = typename Vec16<T>::type;
        V const v = *reinterpret_cast<V const*>(in + 2 * PV * pv);
        if constexpr (Vec16<T>::n == 4) {
            x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else {
            x[0] = v.x; x[1] = v.y;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 2 * PV; ++e) x[e] = in[(2 * PV * pv + e) * j.si[3]];
    }
    T y[2 * PV];
#pragma unroll
    for (int k = 0; k < PV; ++k) {
        if (!j.rotate) {
            y[2 * k] = x[2 * k];
            y[2 * k + 1] = x[2 * k + 1];
            continue;
        }
        int64_t const p = pv * PV + k;
        T const c = cosT[pos * a.cs0 + p * a.cs1];
        T const s = sinT[pos * a.ss0 + p * a.ss1];
        T const even = x[2 * k], odd = x[2 * k + 1];
        y[2 * k] = sub_rn(mul_rn(even, c), mul_rn(odd, s));
        y[2 * k + 1] = add_rn(mul_rn(even, s), mul_rn(odd, c));
    }
    if constexpr (VEC) {
        using V = typename Vec16<T>::type;
        V v;
        if constexpr (Vec16<T>::n == 4) {
            v.x = y[0]; v.y = y[1]; v.z = y[2]; v.w = y[3];
        } else {
            v.x = y[0]; v.y = y[1];
        }
        *reinterpret_cast<V*>(out + 2 * PV * pv) = v;
    } else {
#pragma unroll
        for (int e = 0; e < 2 * PV; ++e) out[(2 * PV * pv + e) * j.so[3]] = y[e];
    }
}

// Division of n < 2^31 by an invariant d >= 1 as a multiply and a shift
// (Granlund and Montgomery, "Division by invariant integers using
// multiplication", 1994): with l = ceil(log2 d) and m = ceil(2^(31+l) / d),
// which fits in 32 bits, n / d = (n * m) >> (31 + l) for every n < 2^31.
struct FastDiv {
    uint32_t d, m, shift;
    static FastDiv make(uint32_t d) {
        uint32_t l = 0;
        while ((uint64_t{1} << l) < d) ++l;
        uint64_t const num = uint64_t{1} << (31 + l);
        return FastDiv{d, static_cast<uint32_t>((num + d - 1) / d), 31 + l};
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        return static_cast<uint32_t>((static_cast<uint64_t>(n) * m) >> shift);
    }
};

// The aligned path when every index fits in 31 bits (the normal case): the
// flat item index splits into (a0, a1, a2, pair-vector) with three FastDiv
// steps instead of three 64-bit divisions (which made the kernel
// instruction-bound), and the PV cos/sin entries of an item are one vector
// load each when the tables allow it.
struct RopeFast {
    FastDiv npv[2], e2[2], e1[2];
    int tab_vec;  // cos/sin entries of one item contiguous and 8-byte aligned (fp32 only)
};

template <typename T, int PV>
__device__ __forceinline__ void rope_item_fast(RopeArgs const& a, RopeJob const& j, int jk, RopeFast const& f,
                                               uint32_t flat) {
    uint32_t const r = f.npv[jk].div(flat);
    uint32_t const pv = flat - r * f.npv[jk].d;
    uint32_t const r2 = f.e2[jk].div(r);
    uint32_t const a2 = r - r2 * f.e2[jk].d;
    uint32_t const a0 = f.e1[jk].div(r2);
    uint32_t const a1 = r2 - a0 * f.e1[jk].d;
    int64_t const tok = a.layout == ANN_LAYOUT_BTHD ? a1 : a2;
    int64_t const pos = a.pos_off + tok;
    using V = typename Vec16<T>::type;
    T const* in = static_cast<T const*>(j.in) + a0 * j.si[0] + a1 * j.si[1] + a2 * j.si[2];
    T* out = static_cast<T*>(j.out) + a0 * j.so[0] + a1 * j.so[1] + a2 * j.so[2];
    V const v = *reinterpret_cast<V const*>(in + 2 * PV * static_cast<int64_t>(pv));
    T x[2 * PV];
    if constexpr (PV == 2) {
        x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    } else {
        x[0] = v.x; x[1] = v.y;
    }
    T y[2 * PV];
    if (!j.rotate) {  // a copied job (V of kvCacheAppend) may come with no tables at all
#pragma unroll
        for (int e = 0; e < 2 * PV; ++e) y[e] = x[e];
    } else {
        T c[PV], sn[PV];
        T const* cosT = static_cast<T const*>(a.cos);
        T const* sinT = static_cast<T const*>(a.sin);
        int64_t const p0 = static_cast<int64_t>(pv) * PV;
        bool done = false;
        if constexpr (PV == 2 && sizeof(T) == 4) {
            if (f.tab_vec) {
                float2 const cc = *reinterpret_cast<float2 const*>(cosT + pos * a.cs0 + p0);
                float2 const ss = *reinterpret_cast<float2 const*>(sinT + pos * a.ss0 + p0);
                c[0] = cc.x; c[1] = cc.y; sn[0] = ss.x; sn[1] = ss.y;
                done = true;
            }
        }
        if (!done) {
#pragma unroll
            for (int k = 0; k < PV; ++k) {
                c[k] = cosT[pos * a.cs0 + (p0 + k) * a.cs1];
                sn[k] = sinT[pos * a.ss0 + (p0 + k) * a.ss1];
            }
        }
#pragma unroll
        for (int k = 0; k < PV; ++k) {
            T const even = x[2 * k], odd = x[2 * k + 1];
            y[2 * k] = sub_rn(mul_rn(even, c[k]), mul_rn(odd, sn[k]));
            y[2 * k + 1] = add_rn(mul_rn(even, sn[k]), mul_rn(odd, c[k]));
        }
    }
    V w;
    if constexpr (PV == 2) {
        w.x = y[0]; w.y = y[1]; w.z = y[2]; w.w = y[3];
    } else {
        w.x = y[0]; w.y = y[1];
    }
    *reinterpret_cast<V*>(out + 2 * PV * static_cast<int64_t>(pv)) = w;
}

template <typename T, int PV>
__global__ void __launch_bounds__(256) rope_kernel_fast(RopeArgs a, RopeFast f) {
    uint32_t const n0 = static_cast<uint32_t>(a.job[0].items);
    uint32_t const total = n0 + (a.njobs > 1 ? static_cast<uint32_t>(a.job[1].items) : 0u);  // < 2^31
    uint32_t const step = gridDim.x * blockDim.x;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        if (i < n0)
            rope_item_fast<T, PV>(a, a.job[0], 0, f, i);
        else
            rope_item_fast<T, PV>(a, a.job[1], 1, f, i - n0);
    }
}

template <typename T, int PV, bool VEC>
__global__ void __launch_bounds__(256) rope_kernel(RopeArgs a) {
    int64_t const total = a.job[0].items + (a.njobs > 1 ? a.job[1].items : 0);
    int64_t const step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += step) {
        if (i < a.job[0].items)
            rope_item<T, PV, VEC>(a, a.job[0], i);
        else
            rope_item<T, PV, VEC>(a, a.job[1], i - a.job[0].items);
    }
}

// validateRopeShape (rope.hpp:21-46), with the coverage check on the layout's
// real token axis (the reference tests axis 1 for every rank-4 tensor).
template <typename T>
int validate(const Dims& in, const Dims& out, const Dims& c, const Dims& s, int layout, uint32_t off) {
    if (!same_extents(in, out)) return fail(ANN_EINVAL, "rope shape mismatch.");
    if (in.rank != 4) return fail(ANN_EINVAL, "rope expects a rank-4 BTHD or BHTD tensor.");
    if (layout != ANN_LAYOUT_BTHD && layout != ANN_LAYOUT_BHTD) return fail(ANN_EINVAL, "rope layout is invalid.");
    int64_t const headDim = in.ext[3];
    if (headDim % 2 != 0) return fail(ANN_EINVAL, "rope requires an even head dimension.");
    if (!same_extents(c, s)) return fail(ANN_EINVAL, "rope cosine/sine table shape mismatch.");
    if (c.rank != 2) return fail(ANN_EINVAL, "rope tables must be rank 2 [positions, headDim/2].");
    if (c.ext[1] != headDim / 2) return fail(ANN_EINVAL, "rope table pair count mismatch.");
    int64_t const tokens = layout == ANN_LAYOUT_BTHD ? in.ext[1] : in.ext[2];
    if (static_cast<int64_t>(off) + tokens > c.ext[0])
        return fail(ANN_EINVAL, "rope table does not cover requested positions.");
    return ANN_OK;
}

template <typename T>
void make_job(RopeJob& j, const Dims& in, const Dims& out, int pv) {
    j.in = in.data;
    j.out = out.data;
    j.e0 = in.ext[0];
    j.e1 = in.ext[1];
    j.e2 = in.ext[2];
    j.npv = in.ext[3] / 2 / pv;
    for (int i = 0; i < 4; ++i) {
        j.si[i] = in.str[i];
        j.so[i] = out.str[i];
    }
    j.items = j.e0 * j.e1 * j.e2 * j.npv;
    j.rotate = 1;
}

template <typename T>
bool vec_ok(const Dims& in, const Dims& out) {
    constexpr int NV = Vec16<T>::n;
    if (in.str[3] != 1 || out.str[3] != 1 || in.ext[3] % NV != 0) return false;
    if (!aligned(in.data, 16) || !aligned(out.data, 16)) return false;
    for (int i = 0; i < 3; ++i)
        if ((in.str[i] * sizeof(T)) % 16 != 0 || (out.str[i] * sizeof(T)) % 16 != 0) return false;
    return true;
}

template <typename T>
int launch(ann_stream stream, const Dims* ins, const Dims* outs, int njobs, const Dims& c, const Dims& s, int layout,
           uint32_t off, const int* rotate = nullptr) {
    constexpr int PVV = Vec16<T>::n / 2;  // pairs per 16-byte vector
    bool vec = true;
    for (int k = 0; k < njobs; ++k) vec = vec && vec_ok<T>(ins[k], outs[k]);
    int const pv = vec ? PVV : 1;
    RopeArgs a{};
    a.njobs = 0;
    for (int k = 0; k < njobs; ++k) {
        if (ins[k].numel() == 0) continue;
        make_job<T>(a.job[a.njobs], ins[k], outs[k], pv);
        if (rotate != nullptr) a.job[a.njobs].rotate = rotate[k];
        ++a.njobs;
    }
    if (a.njobs == 0) return ANN_OK;
    a.cos = c.data;
    a.sin = s.data;
    a.cs0 = c.str[0];
    a.cs1 = c.str[1];
    a.ss0 = s.str[0];
    a.ss1 = s.str[1];
    a.layout = layout;
    a.pos_off = off;
    int64_t const total = a.job[0].items + (a.njobs > 1 ? a.job[1].items : 0);
    int const grid = grid_for(total, 256);
    bool fast = vec && total < (int64_t{1} << 31);
    for (int k = 0; fast && k < a.njobs; ++k)
        fast = a.job[k].npv >= 1 && a.job[k].e2 >= 1 && a.job[k].e1 >= 1;
    if (fast) {
        RopeFast f{};
        for (int k = 0; k < a.njobs; ++k) {
            f.npv[k] = FastDiv::make(static_cast<uint32_t>(a.job[k].npv));
            f.e2[k] = FastDiv::make(static_cast<uint32_t>(a.job[k].e2));
            f.e1[k] = FastDiv::make(static_cast<uint32_t>(a.job[k].e1));
        }
        f.tab_vec = sizeof(T) == 4 && a.cs1 == 1 && a.ss1 == 1 && a.cs0 % 2 == 0 && a.ss0 % 2 == 0 &&
                    aligned(a.cos, 8) && aligned(a.sin, 8);
        rope_kernel_fast<T, PVV><<<grid, 256, 0, as_stream(stream)>>>(a, f);
    } else if (vec)
        rope_kernel<T, PVV, true><<<grid, 256, 0, as_stream(stream)>>>(a);
    else
        rope_kernel<T, 1, false><<<grid, 256, 0, as_stream(stream)>>>(a);
    return check_launch("rope");
}

template <typename T>
int rope(ann_stream stream, const ann_view* in_v, const ann_view* c_v, const ann_view* s_v, const ann_view* out_v,
         int layout, uint32_t off) {
    Dims in, out, c, s;
    ANN_TRY(to_dims(in_v, sizeof(T), "rope input", in));
    ANN_TRY(to_dims(out_v, sizeof(T), "rope output", out));
    ANN_TRY(to_dims(c_v, sizeof(T), "rope cosine table", c));
    ANN_TRY(to_dims(s_v, sizeof(T), "rope sine table", s));
    ANN_TRY(validate<T>(in, out, c, s, layout, off));
    return launch<T>(stream, &in, &out, 1, c, s, layout, off);
}

template <typename T>
int rope_inplace(ann_stream stream, const ann_view* q_v, const ann_view* k_v, const ann_view* c_v,
                 const ann_view* s_v, int layout, uint32_t off) {
    Dims t[2], c, s;
    ANN_TRY(to_dims(q_v, sizeof(T), "ropeInPlace q", t[0]));
    int n = 1;
    if (k_v != nullptr) {
        ANN_TRY(to_dims(k_v, sizeof(T), "ropeInPlace k", t[1]));
        n = 2;
    }
    ANN_TRY(to_dims(c_v, sizeof(T), "rope cosine table", c));
    ANN_TRY(to_dims(s_v, sizeof(T), "rope sine table", s));
    for (int k = 0; k < n; ++k) ANN_TRY(validate<T>(t[k], t[k], c, s, layout, off));
    return launch<T>(stream, t, t, n, c, s, layout, off);
}

// k_new, v_new: BTHD [B, Tn, Hkv, D]; k_cache, v_cache: BHTD [B, Hkv, Tcap, D];
// rows go to cache tokens [position, position + Tn). cos/sin NULL: no rotation.
template <typename T>
int kv_cache_append(ann_stream stream, const ann_view* kn_v, const ann_view* vn_v, const ann_view* kc_v,
                    const ann_view* vc_v, const ann_view* c_v, const ann_view* s_v, uint32_t position) {
    Dims kn, vn, kc, vc, c, s;
    ANN_TRY(to_dims(kn_v, sizeof(T), "kvCacheAppend k_new", kn));
    ANN_TRY(to_dims(vn_v, sizeof(T), "kvCacheAppend v_new", vn));
    ANN_TRY(to_dims(kc_v, sizeof(T), "kvCacheAppend k_cache", kc));
    ANN_TRY(to_dims(vc_v, sizeof(T), "kvCacheAppend v_cache", vc));
    if (kn.rank != 4 || vn.rank != 4 || kc.rank != 4 || vc.rank != 4)
        return fail(ANN_EINVAL, "kvCacheAppend expects rank-4 BTHD rows and BHTD caches.");
    if (!same_extents(kn, vn) || !same_extents(kc, vc)) return fail(ANN_EINVAL, "kvCacheAppend K/V shape mismatch.");
    if (kc.ext[0] != kn.ext[0] || kc.ext[1] != kn.ext[2] || kc.ext[3] != kn.ext[3])
        return fail(ANN_EINVAL, "kvCacheAppend: rows %s do not match the cache %s.", extents_str(kn).c_str(),
                    extents_str(kc).c_str());
    if (static_cast<int64_t>(position) + kn.ext[1] > kc.ext[2])
        return fail(ANN_EINVAL, "kvCacheAppend past the cache capacity (%lld + %lld > %lld).",
                    static_cast<long long>(position), static_cast<long long>(kn.ext[1]),
                    static_cast<long long>(kc.ext[2]));
    bool const rope = c_v != nullptr || s_v != nullptr;
    if (rope) {
        if (c_v == nullptr || s_v == nullptr) return fail(ANN_EINVAL, "kvCacheAppend needs both RoPE tables.");
        ANN_TRY(to_dims(c_v, sizeof(T), "rope cosine table", c));
        ANN_TRY(to_dims(s_v, sizeof(T), "rope sine table", s));
        ANN_TRY(validate<T>(kn, kn, c, s, ANN_LAYOUT_BTHD, position));
    }
    if (kn.numel() == 0) return ANN_OK;
    // the caches seen in the rows' axis order (B, T, H, D), starting at `position`
    Dims outs[2] = {kc, vc};
    for (Dims* o : {&outs[0], &outs[1]}) {
        Dims const cache = *o;
        o->data = static_cast<T*>(cache.data) + static_cast<int64_t>(position) * cache.str[2];
        o->ext[0] = kn.ext[0], o->ext[1] = kn.ext[1], o->ext[2] = kn.ext[2], o->ext[3] = kn.ext[3];
        o->str[0] = cache.str[0], o->str[1] = cache.str[2], o->str[2] = cache.str[1], o->str[3] = cache.str[3];
    }
    Dims const ins[2] = {kn, vn};
    int const rotate[2] = {rope ? 1 : 0, 0};
    return launch<T>(stream, ins, outs, 2, c, s, ANN_LAYOUT_BTHD, position, rotate);
}

}  // namespace
}  // namespace ann

extern "C" {

int ann_kv_cache_append_f32(ann_stream st, const ann_view* k_new, const ann_view* v_new, const ann_view* k_cache,
                            const ann_view* v_cache, const ann_view* cos_table, const ann_view* sin_table,
                            uint32_t position) {
    ANN_API_BEGIN
    return ann::kv_cache_append<float>(st, k_new, v_new, k_cache, v_cache, cos_table, sin_table, position);
    ANN_API_END
}
int ann_kv_cache_append_f64(ann_stream st, const ann_view* k_new, const ann_view* v_new, const ann_view* k_cache,
                            const ann_view* v_cache, const ann_view* cos_table, const ann_view* sin_table,
                            uint32_t position) {
    ANN_API_BEGIN
    return ann::kv_cache_append<double>(st, k_new, v_new, k_cache, v_cache, cos_table, sin_table, position);
    ANN_API_END
}

int ann_rope_f32(ann_stream st, const ann_view* in, const ann_view* c, const ann_view* s, const ann_view* out,
                 int32_t layout, uint32_t off) {
    ANN_API_BEGIN
    return ann::rope<float>(st, in, c, s, out, layout, off);
    ANN_API_END
}
int ann_rope_f64(ann_stream st, const ann_view* in, const ann_view* c, const ann_view* s, const ann_view* out,
                 int32_t layout, uint32_t off) {
    ANN_API_BEGIN
    return ann::rope<double>(st, in, c, s, out, layout, off);
    ANN_API_END
}
int ann_rope_inplace_f32(ann_stream st, const ann_view* q, const ann_view* k, const ann_view* c, const ann_view* s,
                         int32_t layout, uint32_t off) {
    ANN_API_BEGIN
    return ann::rope_inplace<float>(st, q, k, c, s, layout, off);
    ANN_API_END
}
int ann_rope_inplace_f64(ann_stream st, const ann_view* q, const ann_view* k, const ann_view* c, const ann_view* s,
                         int32_t layout, uint32_t off) {
    ANN_API_BEGIN
    return ann::rope_inplace<double>(st, q, k, c, s, layout, off);
    ANN_API_END
}

}  // extern "C"
