from ._native import native, available, check_error, NativeUnavailable
