from ferrite.serving.engine import Engine, ServeConfig

__all__ = ["Engine", "ServeConfig"]
