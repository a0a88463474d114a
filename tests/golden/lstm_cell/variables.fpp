#:set architecture = [('Transpose', ['input'], [[2, 1, 3]]), ('LSTM', ['input', 'hidden_state', 'cell_state'], ['output0'], [0])]
#:set inputs = [['output0', 4]]
#:set trueInputs = [['input', [1, 2, 5]], ['hidden_state', [1, 1, 2]], ['cell_state', [1, 1, 2]]]
#:set outShape = [['output', [1, 1, 2]]]
#:set outputs = {'output': 'cell_state'}
