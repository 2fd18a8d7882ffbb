"""Model conversion for the inference hot path (memfast/nn/conversion.py:26-250).

``convert_model`` replaces selected ``nn.Linear`` / ``nn.Conv2d`` modules with
``AnalogLinear`` / ``AnalogConv2d``.  What it keeps from the reference is the
user-visible contract: ``include``/``exclude`` select module paths with their
subtrees (exclusion wins, ``""`` is the root), a module reachable under several
paths converts only if every one of its paths is selected, existing analog
layers are atomic and keep their programming, and Llama models that gain
analog linears run with ``pretraining_tp = 1`` (their tensor-partitioned MLP
reads ``.weight`` directly and would bypass the analog layers).
Hardware-aware training conversion and recurrent layers are outside this
engine's scope and raise ``NotImplementedError``.
"""

import copy

from torch import nn

from ..simulator import AnalogMatrix
from .convolution import AnalogConv2d
from .linear import AnalogLinear

_ANALOG = (AnalogMatrix, AnalogConv2d)
_CONVERTIBLE = (nn.Linear, nn.Conv2d)
_RECURRENT = (nn.RNNCell, nn.RNN, nn.GRUCell, nn.GRU)


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


def _within(name, paths):
    """Whether module path ``name`` lies in the subtree of one of ``paths``."""
    return any(path == "" or name == path or name.startswith(path + ".") for path in paths)


class _Plan:
    """Which modules of one model convert, and the conversion itself."""

    def __init__(self, model, simulator, include, exclude):
        self.simulator = simulator
        self.include = None if include is None else _selection_paths(include, "include")
        self.exclude = _selection_paths(exclude, "exclude")
        self._check_paths(dict(model.named_modules(remove_duplicate=False)))

    def _check_paths(self, modules):
        for label, paths in (("included", self.include or set()), ("excluded", self.exclude)):
            unknown = paths - modules.keys()
            if unknown:
                raise ValueError(f"unknown {label} modules: {sorted(unknown)}")
            for path in paths:
                parts = path.split(".")
                ancestors = (".".join(parts[:depth]) for depth in range(len(parts)))
                for ancestor in ancestors:
                    if ancestor != path and isinstance(modules[ancestor], _ANALOG):
                        raise ValueError(f"{path}: selection inside a converted layer is unsupported; "
                                         f"select its path {ancestor!r}")

    def decide(self, target):
        """Sort the (copied) model's modules by identity: excluded, selected, and the
        internals of existing analog layers, which are never touched."""
        paths = {}
        for name, module in target.named_modules(remove_duplicate=False):
            paths.setdefault(id(module), []).append(name)
        self.excluded = {key for key, names in paths.items() if any(_within(n, self.exclude) for n in names)}
        self.selected = {key for key, names in paths.items() if key not in self.excluded and
                         (self.include is None or all(_within(n, self.include) for n in names))}
        self.internal = {id(child) for module in target.modules() if isinstance(module, _ANALOG)
                         for child in module.modules() if child is not module}

    def check_modules(self, target):
        simulator = self.simulator
        for name, module in target.named_modules():
            if isinstance(module, AnalogMatrix) and module.simulator.device != simulator.device:
                raise ValueError(f"{name}: existing analog matrices are bound to their simulator device")
            if id(module) in self.internal or id(module) not in self.selected:
                continue
            if isinstance(module, _RECURRENT):
                raise NotImplementedError(f"{name}: recurrent layers are outside memfast_b200's scope")
            if isinstance(module, nn.Conv2d) and isinstance(module.padding, str):
                raise ValueError(f"{name}: numeric Conv2d padding is required")
            if isinstance(module, _ANALOG):
                for child in module.modules():
                    if isinstance(child, AnalogMatrix) and (child.config != simulator.config
                                                            or child.simulator.mode != simulator.mode):
                        raise ValueError(f"{name}: reconversion requires matching physical config and mode")

    def convert(self, module, name, done):
        key = id(module)
        if key in self.excluded or isinstance(module, _ANALOG):
            return module
        if isinstance(module, _CONVERTIBLE) and key not in self.selected:
            return module
        if key in done:
            return done[key]
        if isinstance(module, nn.Linear):
            done[key] = AnalogLinear(module, self.simulator, name=name or "linear")
        elif isinstance(module, nn.Conv2d):
            done[key] = AnalogConv2d(module, self.simulator, name=name or "conv")
        else:
            # A container: converted in place, child by child (shared children once).
            done[key] = module
            for attr, child in list(module._modules.items()):
                if child is not None:
                    setattr(module, attr, self.convert(child, f"{name}.{attr}" if name else attr, done))
            _single_partition_llama(module)
        return done[key]


def _single_partition_llama(module):
    """Llama's pretraining_tp > 1 path slices ``.weight`` of the MLP projections itself
    (bypassing their forward); a Llama subtree holding analog linears needs 1."""
    config = getattr(module, "config", None)
    if getattr(config, "model_type", None) == "llama" and getattr(config, "pretraining_tp", 1) > 1 and \
            any(isinstance(child, AnalogLinear) for child in module.modules()):
        config.pretraining_tp = 1


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
    plan = _Plan(model, simulator, include, exclude)
    target = model if inplace else copy.deepcopy(model)
    plan.decide(target)
    plan.check_modules(target)
    target.to(simulator.device)
    return plan.convert(target, "", {}).eval().requires_grad_(False)


def reset_read_events(model, event=0):
    """Replay a read event across all programmed matrices."""
    for module in model.modules():
        if isinstance(module, AnalogMatrix):
            module.reset_read(event)
