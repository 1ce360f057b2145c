from .converter import convert_weights, save_tensor, load_tensor
from .loader import load_converted
from .downloader import download_and_convert_weights
