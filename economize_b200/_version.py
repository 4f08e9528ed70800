"""Version of the B200-native economize framework (API level of economize 0.6.0, ``src/economize/_version.py:4``)."""

__version__ = "0.1.0"
#: The economize release whose public API this package mirrors.
API_LEVEL = "0.6.0"
