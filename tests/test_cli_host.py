"""Host logic of the stories-generate mirror (cmd/stories-generate-go/main.go:120-161): prompt
parsing and Go's duration text."""
import pytest

from ane.cmd.stories_generate import go_duration, parse_token_list


def test_parse_token_list_rules():
    assert parse_token_list("") == [1] and parse_token_list("  ") == [1]
    assert parse_token_list("1, 5 ,,9") == [1, 5, 9]
    assert parse_token_list(",,") == [1]
    with pytest.raises(ValueError, match='token\\[1\\]="x"'):
        parse_token_list("1,x")


def test_go_duration_text():
    assert go_duration(0.0) == "0s"
    assert go_duration(0.0004) == "0s"
    assert go_duration(0.123) == "123ms"
    assert go_duration(1.5) == "1.5s"
    assert go_duration(1.234) == "1.234s"
    assert go_duration(2.0) == "2s"
    assert go_duration(61.25) == "1m1.25s"
    assert go_duration(3723.0) == "1h2m3s"
