"""BrainMind's symbolic memory and conversational routing (crates/brain-core/src/brain_mind.rs:781-1737)."""
from brain_b200.models.brain_mind import BrainMind, levenshtein


def _mind():
    return BrainMind(seed=0)


def test_arithmetic_and_variables():
    bm = _mind()
    assert bm.talk("what is 2 + 3", neural_train=False) == "2 + 3 = 5"
    assert bm.talk("12 divided by 4?", neural_train=False) == "12 / 4 = 3"
    assert bm.talk("7 times 6", neural_train=False) == "7 * 6 = 42"
    assert bm.talk("1.5 plus 1", neural_train=False) == "1.5 + 1 = 2.5"
    assert bm.talk("5 / 0", neural_train=False) == "Division by zero is undefined in standard mathematics."
    bm.facts["gravity"] = "9.81 m/s2"
    assert bm.talk("gravity * 2", neural_train=False) == "gravity * 2 = 9.81 * 2 = 19.62"
    assert bm.talk("x + y", neural_train=False) == "x + y represents the algebraic sum of x and y."


def test_word_problems():
    bm = _mind()
    assert bm.talk("what is 20% of 150?", neural_train=False) == "20% of 150 = 30"
    assert bm.talk("15 percent of 200", neural_train=False) == "15% of 200 = 30"
    assert (bm.talk("if a car drive 60km/h then how much in 5 haurs?", neural_train=False)
            == "At 60 km/h, in 5 hours, the distance traveled is 300 km.")
    assert (bm.talk("a train at 50 mph for 30 minutes", neural_train=False)
            == "At 50 mph, in 30 hours, the distance traveled is 25 miles.")


def test_greetings_names_identity():
    bm = _mind()
    assert bm.talk("ello", neural_train=False).startswith("Hello! I am thinking")
    assert bm.talk("helloo there", neural_train=False).startswith("Hello!")  # Levenshtein 1
    assert bm.talk("my name is Ada.", neural_train=False) == "Nice to meet you, Ada! I will remember your name in my memory."
    assert bm.talk("who am i", neural_train=False) == "You are Ada! My teacher and companion."
    assert bm.talk("hi", neural_train=False).startswith("Hello Ada!")
    assert "3D cubic space" in bm.talk("who are you", neural_train=False)
    assert bm.talk("how are you", neural_train=False).startswith("I am feeling active!")
    assert levenshtein("kitten", "sitting") == 3


def test_learning_facts_and_knowledge_search():
    bm = _mind()
    assert bm.talk("cats purr", neural_train=False) == "cats purr... cats purr"  # newborn imitation
    bm.learn_sentence("a photon is a quantum of light")
    assert bm.facts["photon"] == "photon is a quantum of light"
    assert bm.talk("what is a photon?", neural_train=False) == "photon: photon is a quantum of light"
    assert bm.talk("what is a photons?", neural_train=False) == "photon: photon is a quantum of light"  # fuzzy
    s = bm.teach_text("TYPE: concept\nNAME: entropy\nDEFINITION: a measure of disorder\nunit: J/K\nEND\n"
                      "TYPE: law\nNAME: ohm\nFORMULA: V = I R\nEND\n")
    assert s.facts_indexed >= 5 and s.lines_processed == 9
    assert bm.talk("define entropy", neural_train=False) == "entropy: a measure of disorder"
    assert bm.talk("what is ohm", neural_train=False) == "ohm: V = I R"
    assert bm.facts["concept_unit"] == "J/K" and bm.facts["unit"] == "J/K"
    assert bm.talk("what is zorblax?", neural_train=False) == (
        "I don't know about 'zorblax' yet. Could you explain it to me so I can learn it?")


def test_associations_thoughts_and_pruning(tmp_path):
    bm = _mind()
    bm.learn_sentence("the quantum field is strange")
    for _ in range(3):
        bm.learn_sentence("neural networks learn features")
    bm.facts["x"] = "y"
    assert bm.talk("tell the field story", neural_train=False) == "field is strange"  # association
    assert bm.talk("neural stuff", neural_train=False) == "When I think of neural, it connects to networks and learn."
    assert bm.transitions["neural"]["networks"] == 3.0 and bm.transitions["neural"]["stuff"] == 1.0
    removed = bm.prune_memory(2.0)
    assert removed > 0 and "networks" in bm.transitions["neural"]
    p = str(tmp_path / "m.bn")
    bm.save(p)
    bm2 = BrainMind.load(p)
    assert bm2.transitions == bm.transitions and bm2.facts == bm.facts and bm2.vocab == bm.vocab
