"""CUDA (sm_100a) backend of ViperBench ``cross_entropy`` (forward).

Same signature as ViperBench/cross_entropy/pytorch_impl.py:4-90::

    cross_entropy_fwd(logits, labels, smoothing, logit_scale, lse_square_scale,
                      ignored_index, total_classes, class_start_idx, BLOCK_SIZE,
                      HAS_SMOOTHING, SPLIT) -> (loss, lse, z_loss)

``cross_entropy_bwd(dloss, logits, lse, labels, smoothing, logit_scale,
lse_square_scale, ignored_index, total_classes, class_start_idx, BLOCK_SIZE,
HAS_SMOOTHING)`` mirrors pytorch_impl.py:93-141 and returns dlogits with the
shape and dtype of logits; lse is read as one value per row (flat index r),
as the Triton kernel reads it (triton_impl.py:111).

Each forward output is a float32 tensor of shape [n_rows, n_cols] in the kernel layout
of ViperBench/cross_entropy/triton_impl.py:123-140: the value for row r and
column block cb sits at flat index cb * n_rows + r, for
cb < ceil(n_cols / BLOCK_SIZE). As with the Triton backend the outputs are
allocated with torch.empty, so flat entries past the valid range are not
written (pytorch_impl zero-fills them). Under SPLIT the z_loss entries are 0.
"""
import torch

from .. import _lib

_fast_cross_entropy_fwd = _lib.fast_op("cross_entropy_fwd")


def cross_entropy_fwd(
    logits, labels, smoothing, logit_scale, lse_square_scale,
    ignored_index, total_classes, class_start_idx, BLOCK_SIZE, HAS_SMOOTHING, SPLIT
):
    out = _fast_cross_entropy_fwd(logits, labels, smoothing, logit_scale, lse_square_scale, ignored_index, total_classes,
                   class_start_idx, BLOCK_SIZE, HAS_SMOOTHING, SPLIT)
    if out is not None:  # the C++ fast path took the common case
        return out
    dev = _lib.require_cuda(logits, labels, what="cross_entropy_fwd")
    lcode = _lib.float_code(logits, "cross_entropy_fwd logits")
    if logits.dim() != 2:
        raise ValueError(f"cross_entropy_fwd: logits must be 2-D, got shape {tuple(logits.shape)}")
    if labels.dtype not in _lib.LABEL_CODES:
        raise TypeError(f"cross_entropy_fwd: labels must be int32 or int64, got {labels.dtype}")
    n_rows, n_cols = logits.shape
    if labels.dim() != 1 or labels.shape[0] != n_rows:
        raise ValueError(f"cross_entropy_fwd: labels shape {tuple(labels.shape)} != ({n_rows},)")
    if int(BLOCK_SIZE) <= 0:
        raise ValueError(f"cross_entropy_fwd: BLOCK_SIZE must be positive, got {BLOCK_SIZE}")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    labels = labels.contiguous()
    loss = torch.empty((n_rows, n_cols), dtype=torch.float32, device=logits.device)
    lse = torch.empty((n_rows, n_cols), dtype=torch.float32, device=logits.device)
    z_loss = torch.empty((n_rows, n_cols), dtype=torch.float32, device=logits.device)
    if n_rows == 0 or n_cols == 0:
        return loss, lse, z_loss
    _lib.launch(
        dev, "dslpg_cross_entropy_fwd",
        logits.data_ptr(), labels.data_ptr(), loss.data_ptr(), lse.data_ptr(), z_loss.data_ptr(),
        n_rows, n_cols, logits.stride(0), lcode, _lib.LABEL_CODES[labels.dtype],
        float(smoothing), float(logit_scale), float(lse_square_scale), int(ignored_index),
        float(total_classes), int(class_start_idx), int(BLOCK_SIZE),
        1 if HAS_SMOOTHING else 0, 1 if SPLIT else 0)
    return loss, lse, z_loss


def cross_entropy_bwd(
    dloss, logits, lse, labels, smoothing, logit_scale, lse_square_scale,
    ignored_index, total_classes, class_start_idx, BLOCK_SIZE, HAS_SMOOTHING
):
    dev = _lib.require_cuda(dloss, logits, lse, labels, what="cross_entropy_bwd")
    lcode = _lib.float_code(logits, "cross_entropy_bwd logits")
    dcode = _lib.float_code(dloss, "cross_entropy_bwd dloss")
    if logits.dim() != 2:
        raise ValueError(f"cross_entropy_bwd: logits must be 2-D, got shape {tuple(logits.shape)}")
    if labels.dtype not in _lib.LABEL_CODES:
        raise TypeError(f"cross_entropy_bwd: labels must be int32 or int64, got {labels.dtype}")
    n_rows, n_cols = logits.shape
    if labels.dim() != 1 or labels.shape[0] != n_rows:
        raise ValueError(f"cross_entropy_bwd: labels shape {tuple(labels.shape)} != ({n_rows},)")
    if dloss.dim() != 1 or dloss.shape[0] < n_rows:
        raise ValueError(f"cross_entropy_bwd: dloss must be 1-D with at least {n_rows} entries")
    if lse.numel() < n_rows:
        raise ValueError(f"cross_entropy_bwd: lse needs at least {n_rows} values")
    if int(BLOCK_SIZE) <= 0:
        raise ValueError(f"cross_entropy_bwd: BLOCK_SIZE must be positive, got {BLOCK_SIZE}")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    lse_flat = lse.reshape(-1)
    if lse_flat.dtype != torch.float32:
        raise TypeError(f"cross_entropy_bwd: lse must be float32 (the forward's output), got {lse.dtype}")
    lse_flat = lse_flat.contiguous()
    labels = labels.contiguous()
    dlogits = torch.empty((n_rows, n_cols), dtype=logits.dtype, device=logits.device)
    if n_rows == 0 or n_cols == 0:
        return dlogits
    _lib.launch(
        dev, "dslpg_cross_entropy_bwd",
        dloss.data_ptr(), dcode, dloss.stride(0), logits.data_ptr(), lse_flat.data_ptr(), labels.data_ptr(),
        dlogits.data_ptr(), n_rows, n_cols, logits.stride(0), n_cols, lcode, _lib.LABEL_CODES[labels.dtype],
        float(smoothing), float(logit_scale), float(lse_square_scale), int(ignored_index),
        float(total_classes), int(class_start_idx), 1 if HAS_SMOOTHING else 0)
    return dlogits


def cross_entropy_fwd_bwd(
    logits, labels, dloss, smoothing, logit_scale, lse_square_scale,
    ignored_index, total_classes, class_start_idx, HAS_SMOOTHING
):
    """``cross_entropy_fwd`` with one column block per row (BLOCK_SIZE >= n_cols,
    SPLIT False) followed by ``cross_entropy_bwd`` with ``dloss``, in one pass
    over the logits: for a dloss known before the forward (the gradient of a
    mean or sum of the losses, e.g. ``dloss = full(n_rows, 1 / n_valid)``).

    Returns ``(loss, lse, z_loss, dlogits)``: the first three are 1-D
    ``[n_rows]`` float32 (the forward's values at flat index r), dlogits has the
    logits' shape and dtype. The logits are read from HBM once instead of
    twice (forward, then backward)."""
    dev = _lib.require_cuda(logits, labels, dloss, what="cross_entropy_fwd_bwd")
    lcode = _lib.float_code(logits, "cross_entropy_fwd_bwd logits")
    dcode = _lib.float_code(dloss, "cross_entropy_fwd_bwd dloss")
    if logits.dim() != 2:
        raise ValueError(f"cross_entropy_fwd_bwd: logits must be 2-D, got shape {tuple(logits.shape)}")
    if labels.dtype not in _lib.LABEL_CODES:
        raise TypeError(f"cross_entropy_fwd_bwd: labels must be int32 or int64, got {labels.dtype}")
    n_rows, n_cols = logits.shape
    if labels.dim() != 1 or labels.shape[0] != n_rows:
        raise ValueError(f"cross_entropy_fwd_bwd: labels shape {tuple(labels.shape)} != ({n_rows},)")
    if dloss.dim() != 1 or dloss.shape[0] < n_rows:
        raise ValueError(f"cross_entropy_fwd_bwd: dloss must be 1-D with at least {n_rows} entries")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    labels = labels.contiguous()
    loss = torch.empty(n_rows, dtype=torch.float32, device=logits.device)
    lse = torch.empty(n_rows, dtype=torch.float32, device=logits.device)
    z_loss = torch.empty(n_rows, dtype=torch.float32, device=logits.device)
    dlogits = torch.empty((n_rows, n_cols), dtype=logits.dtype, device=logits.device)
    if n_rows == 0 or n_cols == 0:
        return loss, lse, z_loss, dlogits
    _lib.launch(
        dev, "dslpg_cross_entropy_fwd_bwd",
        logits.data_ptr(), labels.data_ptr(), dloss.data_ptr(), dcode, dloss.stride(0),
        loss.data_ptr(), lse.data_ptr(), z_loss.data_ptr(), dlogits.data_ptr(),
        n_rows, n_cols, logits.stride(0), n_cols, lcode, _lib.LABEL_CODES[labels.dtype],
        float(smoothing), float(logit_scale), float(lse_square_scale), int(ignored_index),
        float(total_classes), int(class_start_idx), 1 if HAS_SMOOTHING else 0)
    return loss, lse, z_loss, dlogits
