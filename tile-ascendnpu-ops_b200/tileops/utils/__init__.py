from tileops.utils.utils import str2dtype

__all__ = ["str2dtype"]
