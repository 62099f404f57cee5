"""Network-level helpers (SpikingJelly ``functional`` contract)."""


def reset_net(net):
    """Call ``reset()`` on every submodule that has one (stateful neurons and
    fused patterns), clearing membrane state between samples."""
    for m in net.modules():
        if m is not net and hasattr(m, "reset") and callable(m.reset):
            m.reset()
    if hasattr(net, "reset") and callable(net.reset):
        net.reset()


def set_step_mode(net, step_mode: str):
    for m in net.modules():
        if hasattr(m, "_step_mode") or hasattr(type(m), "step_mode"):
            try:
                m.step_mode = step_mode
            except (AttributeError, ValueError):
                pass
