from ferrite.model.gpt import GPTConfig, forward, init_params, loss_fn

__all__ = ["GPTConfig", "forward", "init_params", "loss_fn"]
