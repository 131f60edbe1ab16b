"""Run Hugging Face transformers' Mamba-1 mixer on this library's kernels.

The public surface is the reference's (python/arm_scan/patch.py): ``patch()``,
``unpatch()``, ``stats()``.  The design is this module's own:

* One ``_Router`` object owns the installation: it records every attribute it
  replaces (owner, name, original) so that ``unpatch()`` restores exactly
  those, and counts what each call did.
* The replaced ``MambaMixer.slow_forward`` (HF's path whenever the
  ``mamba_ssm`` CUDA kernels are not installed) sorts each call into one of
  three routes -- ``prefill`` (no cache, or the cached prefill of
  ``generate()``), ``decode`` (one token with a warm cache, "has_previous_state"
  cache API) or ``original`` (training, autograd, CPU decode, unknown API) --
  and runs the first two on the GPU.
* The prefill route runs the mixer's middle section on library kernels:
  causal depthwise conv1d + bias + SiLU in one kernel
  (``causal_conv1d_silu``), then the scan with ``dt_proj``'s bias and the
  softplus applied inside the scan kernel (``delta_bias``,
  ``delta_softplus``), so the dt_proj output is never biased or activated in
  torch.  in_proj, x_proj, dt_proj's matmul and out_proj stay torch GEMMs.
* The decode route is one ``selective_state_update`` per layer and token.

Two cache APIs of transformers are recognised from slow_forward's signature:
"cache_position" (prefill iff cache_position spans the conv kernel; caches
through update_conv_state(layer, state, cache_position) and
ssm_states[layer]) and "has_previous_state" (prefill iff the cache has no
state for the layer; update_conv_state(state, layer) and
update_recurrent_state(state, layer)).  Releases without slow_forward but
with a module-level ``mamba_selective_scan`` get that function replaced.
"""

import inspect
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .op import causal_conv1d_silu, kernel_calls, selective_scan, selective_state_update


@dataclass
class _Counters:
    fast_calls: int = 0       # prefill route (and the scan-function replacement)
    decode_calls: int = 0     # decode route
    fallback_calls: int = 0   # original implementation


class _Router:
    def __init__(self):
        self.saved = []        # (owner, name, original)
        self.api = None
        self.counters = _Counters()

    @property
    def active(self):
        return bool(self.saved)

    def replace(self, owner, name, new):
        self.saved.append((owner, name, getattr(owner, name)))
        setattr(owner, name, new)

    def restore(self):
        for owner, name, orig in reversed(self.saved):
            setattr(owner, name, orig)
        self.saved.clear()
        self.api = None


_ROUTER = _Router()


def _cache_api(fn):
    params = inspect.signature(fn).parameters
    if "cache_position" in params:
        return "cache_position"
    if "cache_params" in params:
        return "has_previous_state"
    return None


def _grad_needed(module, x):
    if not torch.is_grad_enabled():
        return False
    return x.requires_grad or any(p.requires_grad for p in module.parameters())


def _route(mixer, x, cache_params, cache_position, api):
    if mixer.training or _grad_needed(mixer, x):
        return "original"
    if cache_params is None:
        return "prefill" if x.is_cuda else "original"
    if api == "cache_position":
        warm = cache_position is None or cache_position.shape[0] != mixer.conv_kernel_size
    else:
        warm = cache_params.has_previous_state(mixer.layer_idx)
    if not warm:
        return "prefill" if x.is_cuda else "original"
    if api == "has_previous_state" and x.shape[1] == 1 and x.is_cuda:
        return "decode"
    return "original"


def _conv_silu(mixer, hidden):
    """The mixer's conv1d + activation: one library kernel when the
    activation is SiLU (Mamba's), else torch."""
    if isinstance(mixer.act, torch.nn.SiLU) or getattr(mixer, "activation", None) == "silu":
        return causal_conv1d_silu(hidden, mixer.conv1d.weight,
                                  mixer.conv1d.bias if mixer.use_conv_bias else None)
    return mixer.act(mixer.conv1d(hidden)[..., :hidden.shape[-1]])


def _prefill(mixer, x, cache_params, cache_position, attention_mask, api):
    seq_len = x.shape[1]
    out_dtype = x.dtype
    hidden, gate = mixer.in_proj(x).transpose(1, 2).chunk(2, dim=1)
    if attention_mask is not None:
        hidden = hidden * attention_mask.unsqueeze(1)
    if cache_params is not None:
        # the conv cache holds the last kernel_size inputs (zero-padded on the left)
        window = F.pad(hidden, (mixer.conv_kernel_size - seq_len, 0))
        if api == "cache_position":
            cache_params.update_conv_state(mixer.layer_idx, window, cache_position)
        else:
            cache_params.update_conv_state(window, mixer.layer_idx)
    u = _conv_silu(mixer, hidden.contiguous())
    if attention_mask is not None:
        u = u * attention_mask.unsqueeze(1)
    proj = mixer.x_proj(u.transpose(1, 2))
    ts, Bm, Cm = torch.split(proj, [mixer.time_step_rank, mixer.ssm_state_size,
                                    mixer.ssm_state_size], dim=-1)
    # dt_proj without its bias: the scan adds it and applies the softplus
    dt_raw = F.linear(ts, mixer.dt_proj.weight).transpose(1, 2)
    y, h_last = selective_scan(u, dt_raw, -torch.exp(mixer.A_log.float()), Bm.transpose(1, 2),
                               Cm.transpose(1, 2), D=mixer.D, z=gate,
                               delta_bias=mixer.dt_proj.bias, delta_softplus=True,
                               return_last_state=True)
    if cache_params is not None:
        if api == "cache_position":
            cache_params.ssm_states[mixer.layer_idx].copy_(h_last)
        else:
            cache_params.update_recurrent_state(h_last.to(out_dtype), mixer.layer_idx)
    return mixer.out_proj(y.transpose(1, 2).to(out_dtype))


def _decode(mixer, x, cache_params, attention_mask):
    """One token with a warm cache ("has_previous_state" API)."""
    out_dtype = x.dtype
    hidden, gate = mixer.in_proj(x).transpose(1, 2).chunk(2, dim=1)
    if attention_mask is not None:
        hidden = hidden * attention_mask.unsqueeze(1)
    layer = mixer.layer_idx
    h = cache_params.layers[layer].recurrent_states.to(torch.float32).contiguous()
    window = cache_params.update_conv_state(hidden, layer).to(mixer.conv1d.weight.device)
    conv = (window * mixer.conv1d.weight[:, 0, :]).sum(-1)
    if mixer.use_conv_bias:
        conv = conv + mixer.conv1d.bias
    u = mixer.act(conv).to(out_dtype)
    if attention_mask is not None:
        u = u * attention_mask[:, -1:]
    ts, Bm, Cm = torch.split(mixer.x_proj(u), [mixer.time_step_rank, mixer.ssm_state_size,
                                                mixer.ssm_state_size], dim=-1)
    y = selective_state_update(h, u, mixer.dt_proj(ts), -torch.exp(mixer.A_log.float()), Bm, Cm,
                               D=mixer.D, z=gate[:, :, -1], dt_softplus=True)
    cache_params.update_recurrent_state(h.to(out_dtype), layer)
    return mixer.out_proj(y.unsqueeze(1).to(out_dtype))


def _install_mixer(modeling_mamba):
    orig = modeling_mamba.MambaMixer.slow_forward
    api = _cache_api(orig)
    if api is None:
        return None
    names = tuple(inspect.signature(orig).parameters)[2:]
    counters = _ROUTER.counters

    def slow_forward(self, input_states, *args, **kwargs):
        kw = dict(zip(names, args), **kwargs)
        cache_params = kw.get("cache_params")
        cache_position = kw.get("cache_position")
        route = _route(self, input_states, cache_params, cache_position, api)
        if route == "prefill":
            counters.fast_calls += 1
            return _prefill(self, input_states, cache_params, cache_position,
                            kw.get("attention_mask"), api)
        if route == "decode":
            counters.decode_calls += 1
            return _decode(self, input_states, cache_params, kw.get("attention_mask"))
        counters.fallback_calls += 1
        return orig(self, input_states, *args, **kwargs)

    _ROUTER.replace(modeling_mamba.MambaMixer, "slow_forward", slow_forward)
    _ROUTER.api = api
    return f"transformers MambaMixer.slow_forward ({api} API)"


def _install_scan_fn(modeling_mamba):
    """Releases with a module-level ``mamba_selective_scan`` (the argument
    list of ``selective_scan``): calls that need no autograd run here."""
    orig = modeling_mamba.mamba_selective_scan
    counters = _ROUTER.counters

    def mamba_selective_scan(hidden_states, dt, A, B, C, D=None, z=None, delta_bias=None,
                             delta_softplus=False, return_last_state=False, **kwargs):
        args = (hidden_states, dt, A, B, C, D, z, delta_bias)
        if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in args):
            counters.fallback_calls += 1
            return orig(hidden_states, dt, A, B, C, D=D, z=z, delta_bias=delta_bias,
                        delta_softplus=delta_softplus, return_last_state=return_last_state,
                        **kwargs)
        counters.fast_calls += 1
        return selective_scan(hidden_states, dt, A, B, C, D=D, z=z, delta_bias=delta_bias,
                              delta_softplus=delta_softplus, return_last_state=return_last_state)

    _ROUTER.replace(modeling_mamba, "mamba_selective_scan", mamba_selective_scan)
    _ROUTER.api = "selective_scan_fn"
    return "transformers mamba_selective_scan (selective_scan_fn API)"


def patch():
    """Send HF Mamba-1's slow path through the library.  Returns the list of
    replaced targets ([] when this transformers release is not recognised);
    calling it again while patched changes nothing."""
    if _ROUTER.active:
        return [f"already patched ({_ROUTER.api} API)"]
    from transformers.models.mamba import modeling_mamba
    target = None
    if hasattr(modeling_mamba.MambaMixer, "slow_forward"):
        target = _install_mixer(modeling_mamba)
    elif hasattr(modeling_mamba, "mamba_selective_scan"):
        target = _install_scan_fn(modeling_mamba)
    if target is None:
        import warnings
        warnings.warn("patch(): no recognised Mamba mixer entry in this transformers release; "
                      "nothing patched")
        return []
    return [target]


def unpatch():
    """Put back everything ``patch()`` replaced.  False if nothing was patched."""
    if not _ROUTER.active:
        return False
    _ROUTER.restore()
    return True


def stats():
    """How calls were routed since import, and the library's kernel-call count."""
    c = _ROUTER.counters
    return {"fast_calls": c.fast_calls, "fallback_calls": c.fallback_calls,
            "decode_calls": c.decode_calls, "kernel_calls": kernel_calls(),
            "patched": _ROUTER.active, "api": _ROUTER.api}
