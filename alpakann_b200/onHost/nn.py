"""alpaka::nn::onHost::nn -- the attention path and the layers around it
(reference: include/alpaka/nn/onHost/nn/{embedding,rms_norm,attention,rope,
softmax,mlp}.hpp).

Same function names, argument order, defaults and error conditions as the
reference; shape errors raise AnnShapeError (a ValueError), the analogue of
std::invalid_argument. `exec` is accepted and ignored.
"""
import ctypes
import enum
import math
from dataclasses import dataclass

import torch

from .._capi import AnnView, check, lib, ref, view
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


def maskedSoftmax(queue, exec, input, mask, output, axis):
    """onHost/nn/softmax.hpp:42-57: softmax along axis of input + mask."""
    check(fn("masked_softmax", suffix(input, mask, output))(handle(queue), ref(input), ref(mask), ref(output),
                                                           int(axis)))


# ---- MLP layers (onHost/nn/mlp.hpp) -----------------------------------------
class Activation(enum.IntEnum):
    """nn::Activation (mlp.hpp:52-58)."""
    none = 0
    relu = 1
    silu = 2
    gelu = 3


@dataclass
class WeightView:
    """mlp.hpp:60-69: a layer weight [in, out]; not copied, not kept alive."""
    view: torch.Tensor


@dataclass
class BiasView:
    """mlp.hpp:71-76: a layer bias [out]."""
    view: torch.Tensor


def _unwrap(t):
    return t.view if isinstance(t, (WeightView, BiasView)) else t


def linear(queue, input, weight, output):
    """mlp.hpp:33-37: output = input . weight (row-major [in, out]), cuBLAS."""
    gemm(queue, input, weight, output)


def linearBias(queue, exec, input, weight, bias, output, activation=Activation.none):
    """mlp.hpp:42-47: output = input . weight + bias, with an optional
    activation fused into the bias pass."""
    check(fn("linear_bias", suffix(input, weight, bias, output))(handle(queue), ref(input), ref(weight), ref(bias),
                                                               int(activation), ref(output)))


def mlpForward(queue, exec, input, weights, biases, *args, workspace=None):
    """mlp.hpp:150-246. mlpForward(queue, exec, input, weights, biases,
    activation, output) or (..., hiddenActivation, lastActivation, output).
    weights / biases: sequences of tensors or WeightView / BiasView."""
    if len(args) == 2:
        hidden, last, output = args[0], args[0], args[1]
    elif len(args) == 3:
        hidden, last, output = args
    else:
        raise TypeError("mlpForward(queue, exec, input, weights, biases, [hidden,] activation, output)")
    ws = [_unwrap(w) for w in weights]
    bs = [_unwrap(b) for b in biases]
    if len(ws) == 0:
        raise_shape("mlpForward: at least one layer is required.")
    if len(ws) != len(bs):
        raise_shape("mlpForward: weights and biases must have the same length.")
    sfx = suffix(input, output, *ws, *bs)
    wv = (AnnView * len(ws))(*[view(w) for w in ws])
    bv = (AnnView * len(bs))(*[view(b) for b in bs])
    wptr = workspace.data_ptr() if workspace is not None else None
    wbytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(fn("mlp_forward", sfx)(handle(queue), ref(input), len(ws), wv, bv, int(hidden), int(last), ref(output),
                                 wptr, wbytes))


def mlpForwardWorkspaceBytes(input, weights, biases, output):
    """Bytes of scratch mlpForward needs for these shapes (0 for one layer)."""
    ws = [_unwrap(w) for w in weights]
    bs = [_unwrap(b) for b in biases]
    wv = (AnnView * max(1, len(ws)))(*[view(w) for w in ws])
    bv = (AnnView * max(1, len(bs)))(*[view(b) for b in bs])
    out = ctypes.c_uint64(0)
    check(lib.ann_mlp_forward_workspace_bytes(ref(input), len(ws), wv, bv, ref(output), input.element_size(),
                                              ctypes.byref(out)))
    return out.value


def decodeLatent(queue, exec, latent, weight, output):
    """mlp.hpp:277-282: output = latent . weight (no bias, no activation)."""
    gemm(queue, latent, weight, output)


def mlp(queue, exec, input, Wgate, Wup, Wdown, output, workspace=None):
    """mlp.hpp:307-337: output = swiglu(input . Wgate, input . Wup) . Wdown."""
    sfx = suffix(input, Wgate, Wup, Wdown, output)
    wptr = workspace.data_ptr() if workspace is not None else None
    wbytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(fn("mlp", sfx)(handle(queue), ref(input), ref(Wgate), ref(Wup), ref(Wdown), ref(output), wptr, wbytes))


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


def attentionDecodeMirror(queue, exec, Q, K, V, out, outMirror, scale=None, queriesPerKvGroup=1, kvLayout=BHTD):
    """attentionDecode whose results are stored through `outMirror`, the NVLink
    multicast address of out's first element, into every rank's copy of the
    output (include/ann_b200.h, multicast outputs); follow it with the buffer's
    barrier on every rank."""
    sfx = suffix(Q, K, V, out)
    if scale is None:
        scale = 1.0 / math.sqrt(Q.shape[3])
    check(fn("attention_decode_mirror", sfx)(handle(queue), ref(Q), ref(K), ref(V), ref(out),
                                             ctypes.c_void_p(int(outMirror)), float(scale), int(queriesPerKvGroup),
                                             int(kvLayout)))


def attentionPrefillMirror(queue, exec, Q, K, V, out, outMirror, scale=None, queriesPerKvGroup=1, kvLayout=BTHD,
                           causal=True):
    """attentionPrefill with the results stored through the multicast address
    `outMirror` into every rank's copy (see attentionDecodeMirror)."""
    sfx = suffix(Q, K, V, out)
    if scale is None:
        scale = 1.0 / math.sqrt(Q.shape[3])
    check(fn("attention_prefill_mirror", sfx)(handle(queue), ref(Q), ref(K), ref(V), ref(out),
                                              ctypes.c_void_p(int(outMirror)), float(scale), int(queriesPerKvGroup),
                                              int(kvLayout), 1 if causal else 0))


def raise_shape(msg):
    from .._capi import ANN_EINVAL, AnnShapeError
    raise AnnShapeError(ANN_EINVAL, msg)
