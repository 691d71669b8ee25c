"""REPL, script runner, project scaffolding and the BrainMind chat commands of the ``brain`` CLI.

Reference: crates/brain-cli/src/repl/mod.rs:26-100 (``eval_line``: ``name = expr`` bindings, bare
expressions, ``:help :vars :clear :quit :exit`` meta commands, one line per statement),
repl/parser.rs:9-60 (``zeros(...)``, ``ones(...)``, ``add/sub/mul(a, b)``, variables, numbers),
script.rs:9-25 (scripts skip blank and ``#`` lines and stop at the first error), init.rs:8-60
(project scaffold), commands/space_cmd.rs:16-200 (``new`` / ``chat`` / ``chatbot`` over a ``.bn``
BrainMind file with ``--teach``).

The expression language here is parsed by a small recursive-descent parser, so calls nest
(``add(mul(a, 2), ones(3))``), and it adds ``randn``, ``matmul``, ``sum``, ``mean``, ``relu``,
``softmax`` and ``transpose``. Tensors live on the GPU when one is present.
"""
from __future__ import annotations

import os
import re
import sys

OK, ERROR, USAGE, IO_ERROR = 0, 1, 2, 3

_TOKEN = re.compile(r"\s*(?:(\d+\.\d*(?:[eE][-+]?\d+)?|\.\d+(?:[eE][-+]?\d+)?|\d+(?:[eE][-+]?\d+)?)|([A-Za-z_]\w*)|(.))")


class ReplError(Exception):
    pass


def _tokens(s: str):
    out = []
    for num, name, ch in _TOKEN.findall(s):
        if num:
            out.append(("num", num))
        elif name:
            out.append(("name", name))
        elif ch.strip():
            out.append(("op", ch))
    return out


class ReplState:
    def __init__(self, device=None, out=None):
        import torch

        self.torch = torch
        self.device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        self.variables: dict = {}
        self.history: list[str] = []
        self.out = out or (lambda s: print(s))
        self.quit = False

    # ---- expression evaluation
    def _call(self, name: str, args: list):
        t = self.torch
        dims = lambda: [int(a.item()) if hasattr(a, "item") else int(a) for a in args]  # noqa: E731
        f = {
            "zeros": lambda: t.zeros(dims(), device=self.device),
            "ones": lambda: t.ones(dims(), device=self.device),
            "randn": lambda: t.randn(dims(), device=self.device),
            "add": lambda: args[0] + args[1],
            "sub": lambda: args[0] - args[1],
            "mul": lambda: args[0] * args[1],
            "div": lambda: args[0] / args[1],
            "matmul": lambda: t.matmul(args[0], args[1]),
            "sum": lambda: args[0].sum(),
            "mean": lambda: args[0].float().mean(),
            "relu": lambda: t.relu(args[0]),
            "softmax": lambda: t.softmax(args[0], -1),
            "transpose": lambda: args[0].transpose(-2, -1),
        }.get(name)
        if f is None:
            raise ReplError(f"unknown function '{name}'")
        need = {"add": 2, "sub": 2, "mul": 2, "div": 2, "matmul": 2, "sum": 1, "mean": 1, "relu": 1, "softmax": 1,
                "transpose": 1}.get(name)
        if need is not None and len(args) != need:
            raise ReplError(f"{name} requires {need} argument{'s' if need > 1 else ''}")
        try:
            return f()
        except ReplError:
            raise
        except Exception as e:  # shape errors and the like
            raise ReplError(f"{name}: {e}") from None

    def eval_expression(self, expr: str):
        toks = _tokens(expr)
        pos = 0

        def peek():
            return toks[pos] if pos < len(toks) else (None, None)

        def expect(v):
            nonlocal pos
            if peek() != ("op", v):
                raise ReplError(f"expected '{v}' in '{expr}'")
            pos += 1

        def term():
            nonlocal pos
            kind, v = peek()
            if kind == "num":
                pos += 1
                return self.torch.tensor(float(v), device=self.device)
            if kind == "op" and v == "-":
                pos += 1
                return -term()
            if kind == "name":
                pos += 1
                if peek() == ("op", "("):
                    pos += 1
                    args = []
                    if peek() != ("op", ")"):
                        args.append(term())
                        while peek() == ("op", ","):
                            pos += 1
                            args.append(term())
                    expect(")")
                    return self._call(v, args)
                if v in self.variables:
                    return self.variables[v]
                raise ReplError(f"Cannot evaluate expression: '{v}' is not defined")
            raise ReplError(f"Cannot evaluate expression: '{expr}'")

        if not toks:
            raise ReplError("empty expression")
        val = term()
        if pos != len(toks):
            raise ReplError(f"Cannot evaluate expression: trailing input in '{expr}'")
        return val

    @staticmethod
    def _shape(t) -> str:
        return "[" + ", ".join(str(d) for d in t.shape) + "]"

    def eval_line(self, line: str) -> None:
        s = line.strip()
        if not s:
            return
        self.history.append(s)
        if s.startswith(":"):
            return self.handle_meta_command(s)
        m = re.match(r"^([A-Za-z_]\w*)\s*=(.*)$", s)
        if m:
            val = self.eval_expression(m.group(2))
            self.variables[m.group(1)] = val
            self.out(f"{m.group(1)} = {self._shape(val)}")
        else:
            val = self.eval_expression(s)
            self.out(f"ans: {self._shape(val)}" + (f" = {val.item():.6g}" if val.numel() == 1 else ""))

    def handle_meta_command(self, cmd: str) -> None:
        if cmd == ":help":
            self.out("REPL Commands: :vars, :clear, :help, :quit, :exit")
        elif cmd == ":vars":
            self.out("Bound Variables:")
            for k, v in self.variables.items():
                self.out(f"  {k}: {self._shape(v)}")
        elif cmd == ":clear":
            self.variables.clear()
            self.out("Environment cleared.")
        elif cmd in (":quit", ":exit"):
            self.out("Goodbye!")
            self.quit = True
        else:
            self.out(f"Unknown REPL command: '{cmd}'")


def run_repl(stdin=None, out=None) -> int:
    st = ReplState(out=out)
    st.out("brain_b200 REPL. Type ':help' for commands, ':quit' to exit.")
    stdin = stdin or sys.stdin
    for line in stdin:
        try:
            st.eval_line(line)
        except ReplError as e:
            st.out(f"error: {e}")
        if st.quit:
            break
    return OK


def run_script(text: str, out=None) -> int:
    st = ReplState(out=out)
    for line in text.splitlines():
        s = line.strip()
        if not s or s.startswith("#"):
            continue
        try:
            st.eval_line(s)
        except ReplError as e:
            st.out(f"Script error: {e}")
            return ERROR
        if st.quit:
            break
    return OK


def scaffold_project(name: str, out=print) -> int:
    """Creates ``name/`` with ``pyproject.toml``, ``brain.toml``, ``src/model.py`` and ``train.py``."""
    out(f"Creating new Brain project '{name}'...")
    try:
        os.makedirs(os.path.join(name, "src"), exist_ok=False)
    except FileExistsError:
        out(f"error: '{name}' already exists")
        return IO_ERROR
    except OSError as e:
        out(f"error: creating project directory: {e}")
        return IO_ERROR
    files = {
        "pyproject.toml": f'[project]\nname = "{name}"\nversion = "0.1.0"\ndependencies = ["brain_b200"]\n',
        "brain.toml": '# brain_b200 project configuration\n[model]\nname = "model"\ndefault_arch = "mlp"\n',
        os.path.join("src", "model.py"): (
            "from brain_b200.nn import Linear, Module, ReLU\n\n\n"
            "class Model(Module):\n"
            "    def __init__(self, n_in=4, hidden=16, n_out=3):\n"
            "        super().__init__()\n"
            "        self.l1, self.act, self.l2 = Linear(n_in, hidden), ReLU(), Linear(hidden, n_out)\n\n"
            "    def forward(self, x):\n"
            "        return self.l2(self.act(self.l1(x)))\n"),
        "train.py": (
            "import torch\n\nfrom brain_b200.train import Batch, TrainerBuilder\nfrom src.model import Model\n\n"
            "x, y = torch.randn(64, 4), torch.randint(0, 3, (64,))\n"
            "trainer = TrainerBuilder().model(Model()).learning_rate(0.1).build()\n"
            "print(trainer.fit([Batch(x, y)], epochs=5))\n"),
    }
    for rel, text in files.items():
        with open(os.path.join(name, rel), "w") as f:
            f.write(text)
    out(f"[ok] project '{name}' created")
    return OK


def space_command(args: list[str], out=print) -> int:
    """``new <brain.bn> [--teach file] [--steps N]`` creates (or loads) and teaches a BrainMind;
    ``chat <brain.bn> [--message M]`` answers one message, or every line of standard input."""
    from ..models.brain_mind import BrainMind

    if not args:
        out("Usage: brain space new <brain.bn> [--teach <file.txt>] | brain space chat <brain.bn>")
        return USAGE
    sub, rest = args[0], args[1:]
    if sub in ("chat", "chatbot"):
        if not rest:
            out("Usage: brain space chatbot <brain.bn>")
            return USAGE
        try:
            mind = BrainMind.load(rest[0])
        except (OSError, ValueError) as e:
            out(f"error: could not load '{rest[0]}': {e}")
            return IO_ERROR
        msgs = [rest[rest.index("--message") + 1]] if "--message" in rest else [ln.strip() for ln in sys.stdin]
        for m in msgs:
            if m:
                out(f"> {m}\n{mind.talk(m)}")
        return OK
    if sub == "new":
        if not rest:
            out("Usage: brain space new <brain.bn> [--teach <file.txt>]")
            return USAGE
        path = rest[0]
        steps = int(rest[rest.index("--steps") + 1]) if "--steps" in rest else 100
        mind = None
        if os.path.exists(path):
            try:
                mind = BrainMind.load(path)
                out(f"[*] Loaded existing brain '{path}'")
            except (OSError, ValueError) as e:
                out(f"warning: could not load existing '{path}': {e}. Creating a new brain.")
        mind = mind or BrainMind()
        if "--teach" in rest:
            f = rest[rest.index("--teach") + 1]
            try:
                summary = mind.teach_file(f, steps=steps)
            except OSError as e:
                out(f"error reading '{f}': {e}")
                return IO_ERROR
            out(f"[*] Taught from '{f}': {summary.lines_processed} lines, {summary.facts_indexed} facts, "
                f"{summary.words_learned} new words, {summary.synapses_upgraded} synapses, "
                f"neural loss {summary.neural_loss:.3f}")
        mind.save(path)
        out(f"[ok] brain saved to '{path}' (BRAIN_BN v1, CRC-32 checked on load)")
        return OK
    out(f"error: unknown space command '{sub}'")
    return USAGE
