"""Deterministic synthetic corpus for the HRM golden tests (written for this project; exercises speaker tags,
brackets, quotes, tabs, apostrophes, digits, long lines and non-ASCII bytes)."""
import random

WORDS = ("river stone light night garden king queen sword letter ship harbor winter summer bread wine "
         "castle tower bridge market silver golden shadow mirror forest valley mountain storm candle "
         "promise secret journey father mother brother sister friend stranger soldier merchant doctor "
         "engine signal kernel memory vector tensor cache router index query answer retrieval").split()
SPEAKERS = ["ROMEO", "JULIET", "KING LEAR", "O'BRIEN", "NURSE", "FIRST WITCH"]
PROMPTS = [
    "who guards the silver bridge at night",
    "What did the merchant promise the king?",
    "why is the tower dark in winter",
    "tensor cache router index query",
    "ROMEO: where is the golden letter",
    "completely unrelated zebra quantum",
    "",
    "the",
    "garden garden garden garden",
    "Fähre über den Fluss bei Nacht",
]


def corpus(n_lines: int = 900, seed: int = 7) -> str:
    r = random.Random(seed)
    out = []
    for i in range(n_lines):
        k = r.randint(3, 40)
        ws = [r.choice(WORDS) for _ in range(k)]
        s = " ".join(ws).capitalize()
        roll = r.random()
        if roll < 0.15:
            s = r.choice(SPEAKERS) + ": " + s
        if roll > 0.85:
            s += " (" + r.choice(WORDS) + ") [" + r.choice(WORDS) + "]"
        if i % 37 == 0:
            s += "\t" + "\"quoted\" it's " + str(i)
        if i % 53 == 0:
            s = s + ". " + " ".join(r.choice(WORDS) for _ in range(60)) + "; done, " + " ".join(WORDS[:20])
        if i % 71 == 0:
            s += " Straße café naïve"
        if i % 29 == 0:
            out.append("   ")
        out.append(s + ("." if r.random() < 0.5 else ""))
    return "\n".join(out) + "\n"
