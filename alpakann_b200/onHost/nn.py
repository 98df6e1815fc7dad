"""alpaka::nn::onHost::nn -- the attention path (reference:
include/alpaka/nn/onHost/nn/{embedding,rms_norm,attention,rope,softmax}.hpp).

Same function names, argument order, defaults and error conditions as the
reference; shape errors raise AnnShapeError (a ValueError), the analogue of
std::invalid_argument. `exec` is accepted and ignored.
"""
import math

import torch

from .._capi import check, lib, ref
from ._common import ext, fn, gemm, handle, suffix, trace

BTHD, BHTD = 0, 1


def embeddingLookup(queue, exec, tokenIds, embedding, output):
    """onHost/nn/embedding.hpp:17-36. tokenIds: uint32 (int32 accepted, same bits)."""
    if tokenIds.dtype not in (torch.int32, torch.uint32):
        raise TypeError("embeddingLookup expects uint32 token ids")
    check(fn("embedding_lookup", suffix(embedding, output))(handle(queue), ref(tokenIds), ref(embedding),
                                                            ref(output)))


def rmsNorm(queue, exec, input, weight, output, epsilon):
    """onHost/nn/rms_norm.hpp:17-35."""
    check(fn("rms_norm", suffix(input, weight, output))(handle(queue), ref(input), ref(weight), ref(output),
                                                        float(epsilon)))


def embeddingRmsNorm(queue, exec, tokenIds, embedding, weight, output, epsilon):
    """embeddingLookup (onHost/nn/embedding.hpp:17-36) followed by rmsNorm
    (onHost/nn/rms_norm.hpp:17-35) in one launch, bit for bit their result."""
    if tokenIds.dtype not in (torch.int32, torch.uint32):
        raise TypeError("embeddingLookup expects uint32 token ids")
    check(fn("embedding_rms_norm", suffix(embedding, weight, output))(handle(queue), ref(tokenIds), ref(embedding),
                                                                      ref(weight), ref(output), float(epsilon)))


def qkvProjection(queue, input, Wq, Wk, Wv, Q, K, V):
    """onHost/nn/attention.hpp:38-52 (three GEMMs on cuBLAS, no exec)."""
    sfx = suffix(input, Wq, Wk, Wv, Q, K, V)
    check(fn("qkv_projection", sfx)(handle(queue), ref(input), ref(Wq), ref(Wk), ref(Wv), ref(Q), ref(K), ref(V)))


def outputProjection(queue, input, Wo, output):
    """onHost/nn/attention.hpp:112-116."""
    gemm(queue, input, Wo, output)


def outputProjectionResidual(queue, input, Wo, residual, output):
    """outputProjection (onHost/nn/attention.hpp:112-116) then ops::add of the
    residual, fused: output = residual + input . Wo (residual may be output)."""
    check(fn("output_projection_residual", suffix(input, Wo, residual, output))(
        handle(queue), ref(input), ref(Wo), ref(residual), ref(output)))


def kvCacheAppend(queue, exec, kNew, vNew, kCache, vCache, position, cosTable=None, sinTable=None):
    """New K/V rows (BTHD [B,Tn,Hkv,D]) into BHTD caches [B,Hkv,Tcap,D] at tokens
    [position, position + Tn); with RoPE tables K is rotated on the way (as
    ropeInPlace). For an LBHTD cache pass the layer's sub-view."""
    sfx = suffix(kNew, vNew, kCache, vCache)
    c = ref(cosTable) if cosTable is not None else None
    s = ref(sinTable) if sinTable is not None else None
    check(fn("kv_cache_append", sfx)(handle(queue), ref(kNew), ref(vNew), ref(kCache), ref(vCache), c, s,
                                     int(position)))


def _split_tail(args, n_tensors):
    tensors = args[:n_tensors]
    tail = list(args[n_tensors:])
    layout = int(tail[0]) if len(tail) > 0 else BTHD
    offset = int(tail[1]) if len(tail) > 1 else 0
    return tensors, layout, offset


def rope(queue, exec, *args, layout=None, positionOffset=None):
    """onHost/nn/rope.hpp:49-86.
    rope(queue, exec, in, cosTable, sinTable, out, layout=BTHD, positionOffset=0)
    rope(queue, exec, q, k, cosTable, sinTable, outQ, outK, layout=BTHD, positionOffset=0)"""
    n = sum(1 for a in args if isinstance(a, torch.Tensor))
    tensors, lay, off = _split_tail(args, n)
    lay = lay if layout is None else int(layout)
    off = off if positionOffset is None else int(positionOffset)
    if n == 4:
        x, c, s, out = tensors
        check(fn("rope", suffix(x, c, s, out))(handle(queue), ref(x), ref(c), ref(s), ref(out), lay, off))
    elif n == 6:
        q, k, c, s, oq, ok = tensors
        rope(queue, exec, q, c, s, oq, lay, off)
        rope(queue, exec, k, c, s, ok, lay, off)
    else:
        raise TypeError("rope takes 4 or 6 tensors")


def ropeInPlace(queue, exec, *args, layout=None, positionOffset=None):
    """onHost/nn/rope.hpp:96-135, one launch for q and k together.
    ropeInPlace(queue, exec, tensor, cosTable, sinTable, layout=BTHD, positionOffset=0)
    ropeInPlace(queue, exec, q, k, cosTable, sinTable, layout=BTHD, positionOffset=0)"""
    n = sum(1 for a in args if isinstance(a, torch.Tensor))
    tensors, lay, off = _split_tail(args, n)
    lay = lay if layout is None else int(layout)
    off = off if positionOffset is None else int(positionOffset)
    if n == 3:
        t, c, s = tensors
        check(fn("rope_inplace", suffix(t, c, s))(handle(queue), ref(t), None, ref(c), ref(s), lay, off))
    elif n == 4:
        q, k, c, s = tensors
        check(fn("rope_inplace", suffix(q, k, c, s))(handle(queue), ref(q), ref(k), ref(c), ref(s), lay, off))
    else:
        raise TypeError("ropeInPlace takes 3 or 4 tensors")


def attentionScores(queue, exec, Q, K, scores, queriesPerKvGroup=1, kvLayout=BTHD):
    """onHost/nn/attention.hpp:54-81 (unscaled Q.K^T)."""
    if int(queriesPerKvGroup) == 0:
        raise_shape("attentionScores requires queriesPerKvGroup > 0.")
    trace(f"attentionScores q={ext(Q)} k={ext(K)} scores={ext(scores)} queriesPerKvGroup={int(queriesPerKvGroup)}"
          f" layout={'BTHD' if int(kvLayout) == BTHD else 'BHTD'}")
    check(fn("attention_scores", suffix(Q, K, scores))(handle(queue), ref(Q), ref(K), ref(scores),
                                                      int(queriesPerKvGroup), int(kvLayout)))


def attentionApply(queue, exec, probs, values, out, queriesPerKvGroup=1, kvLayout=BTHD):
    """onHost/nn/attention.hpp:83-110."""
    if int(queriesPerKvGroup) == 0:
        raise_shape("attentionApply requires queriesPerKvGroup > 0.")
    trace(f"attentionApply probs={ext(probs)} values={ext(values)} out={ext(out)}"
          f" queriesPerKvGroup={int(queriesPerKvGroup)} layout={'BTHD' if int(kvLayout) == BTHD else 'BHTD'}")
    check(fn("attention_apply", suffix(probs, values, out))(handle(queue), ref(probs), ref(values), ref(out),
                                                           int(queriesPerKvGroup), int(kvLayout)))


def softmax(queue, exec, input, output, axis):
    """onHost/nn/softmax.hpp:26-40."""
    check(fn("softmax", suffix(input, output))(handle(queue), ref(input), ref(output), int(axis)))


def causalSoftmax(queue, exec, input, output, axis, queryAxis, keyAxis):
    """onHost/nn/softmax.hpp:59-80 (top-left causal mask)."""
    check(fn("causal_softmax", suffix(input, output))(handle(queue), ref(input), ref(output), int(axis),
                                                     int(queryAxis), int(keyAxis)))


def attentionDecode(queue, exec, Q, K, V, out, scale=None, queriesPerKvGroup=1, kvLayout=BHTD):
    """Fused decode pipeline attentionScores -> ops::scale -> softmax(axis 3)
    -> attentionApply in one kernel (test/unit/nn/attention.cpp:675-734 is
    the reference composition). scale defaults to 1/sqrt(D)."""
    sfx = suffix(Q, K, V, out)
    if scale is None:
        scale = 1.0 / math.sqrt(Q.shape[3])
    check(fn("attention_decode", sfx)(handle(queue), ref(Q), ref(K), ref(V), ref(out), float(scale),
                                      int(queriesPerKvGroup), int(kvLayout)))


def attentionPrefill(queue, exec, Q, K, V, out, scale=None, queriesPerKvGroup=1, kvLayout=BTHD, causal=True):
    """Fused prefill pipeline attentionScores -> ops::scale -> causalSoftmax
    (top-left mask) or softmax -> attentionApply in one kernel
    (test/unit/nn/attention.cpp:591-651 is the reference composition).
    scale defaults to 1/sqrt(D)."""
    sfx = suffix(Q, K, V, out)
    if scale is None:
        scale = 1.0 / math.sqrt(Q.shape[3])
    check(fn("attention_prefill", sfx)(handle(queue), ref(Q), ref(K), ref(V), ref(out), float(scale),
                                       int(queriesPerKvGroup), int(kvLayout), 1 if causal else 0))


def raise_shape(msg):
    from .._capi import ANN_EINVAL, AnnShapeError
    raise AnnShapeError(ANN_EINVAL, msg)
