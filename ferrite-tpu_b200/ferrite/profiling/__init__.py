from ferrite.profiling.roofline import RooflinePoint, analyze, format_table
from ferrite.profiling.timing import Timing, timeit

__all__ = ["RooflinePoint", "analyze", "format_table", "Timing", "timeit"]
