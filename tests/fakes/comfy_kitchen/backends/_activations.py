import torch.nn.functional as F


def apply_input_act(x, input_act):
    if input_act in (None, "none"):
        return x
    if input_act == "gelu_tanh":
        return F.gelu(x, approximate="tanh")
    if input_act == "gelu":
        return F.gelu(x)
    raise ValueError(input_act)
