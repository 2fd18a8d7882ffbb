"""Model conversion (memfast/nn/conversion.py:26-250) for the inference hot path.

``convert_model`` replaces selected ``nn.Linear`` / ``nn.Conv2d`` modules with
``AnalogLinear`` / ``AnalogConv2d`` using the reference's path-selection,
alias and Llama ``pretraining_tp`` rules.  Hardware-aware training conversion
and recurrent layers are outside this engine's scope and raise
``NotImplementedError``.
"""

import copy

from torch import nn

from ..simulator import AnalogMatrix
from .convolution import AnalogConv2d
from .linear import AnalogLinear


def _selection_paths(value, name):
    if isinstance(value, str):
        raise TypeError(f"{name} must be a sequence of module paths")
    try:
        paths = tuple(value)
    except TypeError:
        raise TypeError(f"{name} must be a sequence of module paths") from None
    if any(not isinstance(path, str) for path in paths):
        raise TypeError(f"{name} module paths must be strings")
    return set(paths)


def convert_model(model, simulator, *, include=None, exclude=(), inplace=False, training=False,
                  gradient_mode="quantized"):
    """Convert Linear and Conv2d modules to analog inference on the B200 engine."""
    if not isinstance(model, nn.Module):
        raise TypeError("model must be a PyTorch module")
    if not isinstance(training, bool):
        raise TypeError("training must be a boolean")
    if gradient_mode not in ("quantized", "digital"):
        raise ValueError("gradient_mode must be quantized or digital")
    if training:
        raise NotImplementedError("hardware-aware training conversion is outside memfast_b200's scope")
    included = None if include is None else _selection_paths(include, "include")
    excluded = _selection_paths(exclude, "exclude")
    analog_types = (AnalogMatrix, AnalogConv2d)
    supported = (nn.Linear, nn.Conv2d)
    recurrent = (nn.RNNCell, nn.RNN, nn.GRUCell, nn.GRU)
    by_path = dict(model.named_modules(remove_duplicate=False))
    for label, selection in (("included", included), ("excluded", excluded)):
        missing = (selection or set()) - by_path.keys()
        if missing:
            raise ValueError(f"unknown {label} modules: {sorted(missing)}")
        for path in selection or ():
            parts = path.split(".")
            for depth in range(len(parts)):
                ancestor = ".".join(parts[:depth])
                if ancestor != path and isinstance(by_path[ancestor], analog_types):
                    raise ValueError(
                        f"{path}: selection inside a converted layer is unsupported; select its path {ancestor!r}"
                    )

    def excluded_path(name):
        return any(path == "" or name == path or name.startswith(path + ".") for path in excluded)

    def included_path(name):
        return included is None or any(
            path == "" or name == path or name.startswith(path + ".") for path in included
        )

    target = model if inplace else copy.deepcopy(model)
    aliases = {}
    for name, module in target.named_modules(remove_duplicate=False):
        aliases.setdefault(id(module), []).append(name)
    excluded_ids = {i for i, names in aliases.items() if any(excluded_path(n) for n in names)}
    selected_ids = {
        i for i, names in aliases.items() if i not in excluded_ids and all(included_path(n) for n in names)
    }
    internal_ids = {
        id(child)
        for module in target.modules()
        if isinstance(module, analog_types)
        for child in module.modules()
        if child is not module
    }
    for name, module in target.named_modules():
        if isinstance(module, AnalogMatrix) and module.simulator.device != simulator.device:
            raise ValueError(f"{name}: existing analog matrices are bound to their simulator device")
        if id(module) in internal_ids or id(module) not in selected_ids:
            continue
        if isinstance(module, recurrent):
            raise NotImplementedError(f"{name}: recurrent layers are outside memfast_b200's scope")
        if isinstance(module, nn.Conv2d) and isinstance(module.padding, str):
            raise ValueError(f"{name}: numeric Conv2d padding is required")
        if isinstance(module, analog_types):
            for child in module.modules():
                if isinstance(child, AnalogMatrix) and (
                    child.config != simulator.config or child.simulator.mode != simulator.mode
                ):
                    raise ValueError(f"{name}: reconversion requires matching physical config and mode")
    target.to(simulator.device)
    replacements = {}

    def convert(module, name):
        if id(module) in excluded_ids:
            return module
        if isinstance(module, supported + analog_types) and id(module) not in selected_ids:
            return module
        if isinstance(module, analog_types):
            return module
        if id(module) in replacements:
            return replacements[id(module)]
        if isinstance(module, nn.Linear):
            result = AnalogLinear(module, simulator, name=name or "linear")
        elif isinstance(module, nn.Conv2d):
            result = AnalogConv2d(module, simulator, name=name or "conv")
        else:
            result = module
            replacements[id(module)] = result
            for attr, child in list(module._modules.items()):
                if child is not None:
                    setattr(module, attr, convert(child, f"{name}.{attr}" if name else attr))
            config = getattr(module, "config", None)
            if (
                getattr(config, "model_type", None) == "llama"
                and getattr(config, "pretraining_tp", 1) > 1
                and any(isinstance(child, AnalogLinear) for child in module.modules())
            ):
                # Tensor-partitioned Llama MLPs read .weight directly and would bypass the analog layers.
                config.pretraining_tp = 1
        replacements[id(module)] = result
        return result

    converted = convert(target, "")
    return converted.eval().requires_grad_(False)


def reset_read_events(model, event=0):
    """Replay a read event across all programmed matrices."""
    for module in model.modules():
        if isinstance(module, AnalogMatrix):
            module.reset_read(event)
