"""Route Hugging Face transformers' Mamba-1 mixer through the GPU scan.

Same surface and behaviour as the reference's python/arm_scan/patch.py:
``patch()`` swaps ``MambaMixer.slow_forward`` (the path HF takes whenever the
``mamba_ssm`` CUDA kernels are not installed, on CPU and on GPU alike) for a
transcription of it whose recurrence runs through ``selective_scan`` with
softplus fused into the kernel; ``unpatch()`` restores the original;
``stats()`` reports engagement.  Projections, conv, gating, weights and cache
seeding are left exactly as upstream does them.

slow_forward's signature changed across transformers releases, so the API is
detected at patch time from the original's parameters:
  "cache_position":     slow_forward(self, x, cache_params, cache_position,
                        attention_mask); prefill iff cache_position spans the
                        conv kernel; caches via update_conv_state(layer, state,
                        cache_position) and ssm_states[layer].copy_()
  "has_previous_state": slow_forward(self, x, cache_params, attention_mask);
                        prefill iff not cache_params.has_previous_state(layer);
                        caches via update_conv_state(state, layer) and
                        update_recurrent_state(state, layer)
For releases without slow_forward but with a module-level
``mamba_selective_scan`` that function is wrapped instead.

The kernel handles cache-less forwards and the cached prefill of
``generate()`` (zero initial state).  With the "has_previous_state" API the
decode steps of ``generate()`` also run on the GPU (one
``selective_state_update`` per layer and token; an extension: the reference
falls back for them).  Other decode steps, mamba.py training mode and any
call that needs autograd (the op has no backward) fall back to the original.
"""

import inspect

import torch
import torch.nn.functional as F

from .op import kernel_calls, selective_scan, selective_state_update

_STATE = {"orig": None, "api": None, "arg_names": (), "target": None,
          "fast_calls": 0, "fallback_calls": 0, "decode_calls": 0}


def _detect_api(orig):
    names = list(inspect.signature(orig).parameters)
    if "cache_position" in names:
        return "cache_position"
    if "cache_params" in names:
        return "has_previous_state"
    return None


def _needs_grad(module, x):
    return torch.is_grad_enabled() and (
        x.requires_grad or any(p.requires_grad for p in module.parameters()))


def _mixer_scan_forward(self, input_states, cache_params, cache_position, attention_mask, api):
    """MambaMixer.slow_forward's no-cache / cached-prefill branch with the
    recurrence on the GPU kernel."""
    seq_len = input_states.shape[1]
    dtype = input_states.dtype
    projected_states = self.in_proj(input_states).transpose(1, 2)
    hidden_states, gate = projected_states.chunk(2, dim=1)
    if attention_mask is not None:
        hidden_states = hidden_states * attention_mask.unsqueeze(1)
    if cache_params is not None:
        conv_state = F.pad(hidden_states, (self.conv_kernel_size - hidden_states.shape[-1], 0))
        if api == "cache_position":
            cache_params.update_conv_state(self.layer_idx, conv_state, cache_position)
        else:
            cache_params.update_conv_state(conv_state, self.layer_idx)
    hidden_states = self.act(self.conv1d(hidden_states)[..., :seq_len])
    if attention_mask is not None:
        hidden_states = hidden_states * attention_mask.unsqueeze(1)
    ssm_parameters = self.x_proj(hidden_states.transpose(1, 2))
    time_step, B, C = torch.split(
        ssm_parameters, [self.time_step_rank, self.ssm_state_size, self.ssm_state_size], dim=-1)
    # raw dt_proj output; softplus runs inside the kernel
    discrete_time_step = self.dt_proj(time_step).transpose(1, 2)
    A = -torch.exp(self.A_log.float())
    scan_output, last_state = selective_scan(
        hidden_states, discrete_time_step, A, B.transpose(1, 2), C.transpose(1, 2),
        D=self.D, z=gate, delta_softplus=True, return_last_state=True)
    if cache_params is not None:
        if api == "cache_position":
            cache_params.ssm_states[self.layer_idx].copy_(last_state)
        else:
            cache_params.update_recurrent_state(last_state.to(dtype), self.layer_idx)
    return self.out_proj(scan_output.transpose(1, 2).to(dtype))


def _mixer_decode_forward(self, input_states, cache_params, attention_mask):
    """MambaMixer.slow_forward's decode branch ("has_previous_state" API, one
    token) with the state update on the GPU kernel."""
    # shapes and mask handling exactly as the original's decode branch
    dtype = input_states.dtype
    projected_states = self.in_proj(input_states).transpose(1, 2)
    hidden_states, gate = projected_states.chunk(2, dim=1)
    if attention_mask is not None:
        hidden_states = hidden_states * attention_mask.unsqueeze(1)
    state = cache_params.layers[self.layer_idx].recurrent_states.to(torch.float32).contiguous()
    conv_state = cache_params.update_conv_state(hidden_states, self.layer_idx)
    conv_state = conv_state.to(self.conv1d.weight.device)
    hidden_states = torch.sum(conv_state * self.conv1d.weight[:, 0, :], dim=-1)
    if self.use_conv_bias:
        hidden_states = hidden_states + self.conv1d.bias
    hidden_states = self.act(hidden_states).to(dtype).unsqueeze(-1)  # [batch, intermediate_size, 1]
    if attention_mask is not None:
        hidden_states = hidden_states * attention_mask.unsqueeze(1)
    hidden_states = hidden_states[:, :, -1]
    ssm_parameters = self.x_proj(hidden_states)
    time_step, B, C = torch.split(
        ssm_parameters, [self.time_step_rank, self.ssm_state_size, self.ssm_state_size], dim=-1)
    A = -torch.exp(self.A_log.float())
    y = selective_state_update(state, hidden_states, self.dt_proj(time_step), A, B, C, D=self.D,
                               z=gate[:, :, -1], dt_softplus=True)
    cache_params.update_recurrent_state(state.to(dtype), self.layer_idx)
    return self.out_proj(y.unsqueeze(1).to(dtype))


def _patch_scan_fn(modeling_mamba):
    """Releases exposing a module-level ``mamba_selective_scan`` (same
    argument list as ``selective_scan``): wrap it, falling back to the
    original for calls that need autograd."""
    orig = modeling_mamba.mamba_selective_scan

    def mamba_selective_scan(hidden_states, dt, A, B, C, D=None, z=None, delta_bias=None,
                             delta_softplus=False, return_last_state=False, use_mambapy=False,
                             use_associative_scan=False, **kwargs):
        tensors = (hidden_states, dt, A, B, C)
        needs_grad = torch.is_grad_enabled() and any(
            t.requires_grad for t in (*tensors, D, z, delta_bias) if t is not None)
        if needs_grad:
            _STATE["fallback_calls"] += 1
            return orig(hidden_states, dt, A, B, C, D=D, z=z, delta_bias=delta_bias,
                        delta_softplus=delta_softplus, return_last_state=return_last_state,
                        use_mambapy=use_mambapy, use_associative_scan=use_associative_scan,
                        **kwargs)
        _STATE["fast_calls"] += 1
        return selective_scan(hidden_states, dt, A, B, C, D=D, z=z, delta_bias=delta_bias,
                              delta_softplus=delta_softplus,
                              return_last_state=return_last_state)

    modeling_mamba.mamba_selective_scan = mamba_selective_scan
    _STATE.update(orig=orig, api="selective_scan_fn", target="mamba_selective_scan")
    return ["transformers mamba_selective_scan (selective_scan_fn API)"]


def patch():
    """Route HF Mamba's slow path through the GPU kernel.  Returns the list of
    patched targets ([] if this transformers release is not recognised).
    Idempotent."""
    if _STATE["orig"] is not None:
        return ["transformers MambaMixer.slow_forward (already patched)"]
    from transformers.models.mamba import modeling_mamba
    if not hasattr(modeling_mamba.MambaMixer, "slow_forward"):
        if hasattr(modeling_mamba, "mamba_selective_scan"):
            return _patch_scan_fn(modeling_mamba)
        import warnings
        warnings.warn("patch(): this transformers release has neither MambaMixer.slow_forward "
                      "nor mamba_selective_scan; leaving it unpatched")
        return []
    orig = modeling_mamba.MambaMixer.slow_forward
    api = _detect_api(orig)
    if api is None:
        import warnings
        warnings.warn("patch(): unrecognised MambaMixer.slow_forward signature; "
                      "leaving it unpatched")
        return []
    arg_names = tuple(inspect.signature(orig).parameters)[2:]

    def slow_forward(self, input_states, *args, **kwargs):
        bound = dict(zip(arg_names, args))
        bound.update(kwargs)
        cache_params = bound.get("cache_params")
        cache_position = bound.get("cache_position")
        attention_mask = bound.get("attention_mask")
        use_mambapy = getattr(self, "use_mambapy", False)
        if api == "cache_position":
            is_prefill = cache_params is None or (
                cache_position is not None and cache_position.shape[0] == self.conv_kernel_size)
        else:
            is_prefill = cache_params is None or not cache_params.has_previous_state(
                self.layer_idx)
        if (not is_prefill and api == "has_previous_state" and input_states.shape[1] == 1
                and input_states.device.type == "cuda" and not self.training
                and not _needs_grad(self, input_states)):
            _STATE["decode_calls"] += 1
            return _mixer_decode_forward(self, input_states, cache_params, attention_mask)
        if (use_mambapy and self.training) or not is_prefill or _needs_grad(self, input_states):
            _STATE["fallback_calls"] += 1
            return orig(self, input_states, *args, **kwargs)
        _STATE["fast_calls"] += 1
        return _mixer_scan_forward(self, input_states, cache_params, cache_position,
                                   attention_mask, api)

    modeling_mamba.MambaMixer.slow_forward = slow_forward
    _STATE.update(orig=orig, api=api, arg_names=arg_names, target="slow_forward")
    return [f"transformers MambaMixer.slow_forward ({api} API)"]


def unpatch():
    """Restore the original implementation.  Returns False if not patched."""
    if _STATE["orig"] is None:
        return False
    from transformers.models.mamba import modeling_mamba
    if _STATE.get("target") == "mamba_selective_scan":
        modeling_mamba.mamba_selective_scan = _STATE["orig"]
    else:
        modeling_mamba.MambaMixer.slow_forward = _STATE["orig"]
    _STATE.update(orig=None, api=None, target=None)
    return True


def stats():
    """Engagement counters."""
    return {"fast_calls": _STATE["fast_calls"], "fallback_calls": _STATE["fallback_calls"],
            "decode_calls": _STATE["decode_calls"],
            "kernel_calls": kernel_calls(), "patched": _STATE["orig"] is not None,
            "api": _STATE["api"]}
