"""No-op stand-in for the third-party ``colored`` package (terminal styling).

The reference front-end imports ``stylize``, ``fore``, ``style``, ``Fore`` and
``Style`` only to colour its debug printing.  This stand-in returns text
unchanged so the reference's passes can be imported for fixture generation.
Written from the call sites in the reference (e.g. autodiff/expr/__init__.py:2,
autodiff/context.py:3); it is not a copy of that package.
"""


def stylize(text, *styles, **kwargs):
    return str(text)


def fore(name):
    return ""


def style(name):
    return ""


def back(name):
    return ""


class _Blank:
    def __getattr__(self, name):
        return ""


Fore = _Blank()
Style = _Blank()
Back = _Blank()
